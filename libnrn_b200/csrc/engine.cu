// engine.cu -- a network resident on one GPU, stepped in CUDA graphs.
//
// One step is the reference's sim_step (src/simulation/runner.cpp:95-173)
// with its phases mapped onto kernels:
//   P1+P2  nrn_cuda_deliver: the spikes emitted d steps ago are added into
//          each target's input accumulator (the accumulators were zeroed by
//          the previous update, which consumes them, so P1 is implicit);
//          the history slot of this step is cleared
//   P3+P4  nrn_cuda_pop_step per population: update, spike flags, ids
//          appended to the population's spike history (the compacted
//          SpikeBuffer) and to the raster (P6, when recorded)
//   P5     nrn_cuda_stdp_step per plastic projection, at slow-clock
//          boundaries (step % slow_ratio == 0, Clock::is_slow_boundary,
//          src/simulation/clock.cpp:59-61)
// A chunk of steps is captured once as a CUDA graph whose kernels read the
// step number as *step_base + offset; one small kernel at the end of the
// chunk advances step_base, so the same graph replays for every chunk.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include <nccl.h>

#include "common.cuh"
#include "detmath.cuh"
#include "internal.h"

namespace nrn {

thread_local std::string g_last_error;

namespace {

template <typename T>
nrn_status_t dalloc0(T** p, size_t n, cudaStream_t s) {
    if (n == 0) n = 1;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(NRN_ERR_OOM, "device allocation of " + std::to_string(n * sizeof(T)) + " bytes failed");
    }
    e = cudaMemsetAsync(*p, 0, n * sizeof(T), s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
    return NRN_OK;
}

__global__ void advance_kernel(long long* base, long long by) { *base += by; }

}  // namespace

nrn_status_t fail(nrn_status_t s, const std::string& msg) {
    g_last_error = msg;
    return s;
}

nrn_status_t cuda_fail(cudaError_t e, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return e == cudaErrorMemoryAllocation ? NRN_ERR_OOM : NRN_ERR_CUDA;
}

}  // namespace nrn

using namespace nrn;

struct EnginePop {
    nrn_pop_desc_t d{};
    int32_t n_global = 0;            // population size over all ranks
    int32_t lo = 0;                  // index of this rank's first neuron
    bool cond = false;
    bool owns_isyn = false;
    float* g_exc = nullptr;
    float* g_inh = nullptr;
    float* gin_exc = nullptr;
    float* gin_inh = nullptr;
    // spike history ring of the whole population: [depth][hist_cap]
    int32_t* hist_ids = nullptr;
    int32_t* hist_count = nullptr;
    int32_t hist_cap = 0;
    // send block of this population inside a rank's exchange buffer
    int64_t send_off = 0;
    int32_t send_cap = 0;
    // for projections with walk plasticity: window spike masks and spike steps
    uint32_t* mask = nullptr;        // [n_global]
    int32_t* recent = nullptr;       // [n_global][4] newest four spike steps
    int32_t* ring = nullptr;         // [n][kRing] spike steps of this rank's neurons
    int32_t* cnt = nullptr;          // [n]
    float* drive_buf = nullptr;      // [n] this step's drive, drawn ahead on the side stream
    nrn_spike_stat_t* stats = nullptr;   // [n] spike statistics (when enabled)
    // synapse channels (per-neuron synapse state, nrn_syn_desc_t)
    int32_t n_chan = 0;
    nrn_syn_desc_t chan[NRN_MAX_CHANNELS]{};
    float* chan_in[NRN_MAX_CHANNELS] = {};
    float* chan_s[NRN_MAX_CHANNELS] = {};
    float* chan_r[NRN_MAX_CHANNELS] = {};
    uint8_t* flags = nullptr;        // deterministic delivery: [det_ring][n] spiked at step s
};

struct EngineProj {
    int32_t src_pop = 0, tgt_pop = 0, receptor = 0;
    DevCsr csr;
    bool plastic = false;
    bool clamped = false;
    double stdp[7] = {0};
    float* x_pre = nullptr;
    float* x_post = nullptr;
    bool traces_fused = false;   // both traces advanced by the neuron updates
    bool walk = false;           // updates applied by segment walks (plastic.cu)
    int32_t* seg_last = nullptr;
    float* seg_x = nullptr;
    float* pre_snap = nullptr;   // [pre_depth][n_src] source trace at window ends
    float* post_ring = nullptr;  // [ring_depth][n_tgt] target trace at every step
    unsigned int* work_ctr = nullptr;   // [3] unit counters of the walk launches
    int32_t pre_depth = 1;
};

struct EngineProbe {
    int32_t pop = 0, var = 0, depth = 1;
    float* ring = nullptr;
};

// Row (step % depth) of a probe ring from a population's state variable.
__global__ void probe_kernel(const float* src, int n, float* ring, int depth, long long step_off,
                             const long long* step_base) {
    const long long step = step_off + *step_base;
    float* row = ring + (step % depth) * static_cast<long long>(n);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) row[i] = src[i];
}

constexpr int kRing = 64;           // spike steps kept per neuron
constexpr int kSweepPeriod = 640;   // the sweep looks at every row this often
constexpr int kStale = 480;         // and walks segments not walked for this many steps

struct nrn_engine {
    int device = 0;
    double dt = 1e-4;
    int32_t slow_ratio = 1;
    cudaStream_t stream = nullptr;
    cudaStream_t side = nullptr;          // static delivery, concurrent with the STDP walks
    cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
    std::vector<EnginePop> pops;
    std::vector<EngineProj> projs;
    std::vector<EngineProbe> probes;
    bool finalized = false;
    int32_t depth = 2;
    int64_t step = 0;                     // host mirror of the device step
    int64_t step_high = 0;                // largest step number reached (bounds the raster's steps)
    RasterSortScratch sort_scratch;       // raster sort buffers, kept between reads
    long long* d_step = nullptr;          // device step base
    unsigned long long* d_events = nullptr;   // [2]: static delivery, walks
    unsigned long long* d_raster_count = nullptr;
    int32_t* raster_step = nullptr;
    int32_t* raster_gid = nullptr;
    int64_t raster_cap = 0;
    int64_t spikes_flushed = 0;
    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;   // (window phase of the first step, steps)
    int* d_err = nullptr;                 // device error flag (plasticity, exchange)
    bool use_graphs = true;
    bool det = false;                     // deterministic delivery (nrn_engine_set_deterministic)
    int32_t det_ring = 1;
    bool spike_stats = false;             // per-neuron spike statistics kept
    // partition over GPUs
    int32_t rank = 0, world = 1;
    ncclComm_t comm = nullptr;
    double comm_timeout_s = 120.0;        // bound of every host wait on the communicator
    bool comm_failed = false;             // the communicator was aborted: no further runs
    bool stuck = false;                   // the stream did not drain after an abort
    double max_rate_hz = 200.0;           // sizes the exchange buffers
    // windows (exchange of spikes, STDP trace snapshots)
    bool windows = false;
    int32_t win = 1;
    int32_t* send = nullptr;              // [rank_block]
    int32_t* recv = nullptr;              // [world][rank_block]
    int64_t rank_block = 0;
    int32_t ring_depth = 1;               // steps of target trace kept (walk projections)

    ~nrn_engine() {
        if (device >= 0) cudaSetDevice(device);
        if (stuck) {
            // work still queued on the stream after a communicator abort:
            // freeing would wait for it, so the buffers are left to the process
            comm = nullptr;
            return;
        }
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        for (auto& p : pops) {
            if (p.owns_isyn) cudaFree(p.d.i_syn);
            cudaFree(p.g_exc); cudaFree(p.g_inh); cudaFree(p.gin_exc); cudaFree(p.gin_inh);
            cudaFree(p.hist_ids); cudaFree(p.hist_count);
            cudaFree(p.mask); cudaFree(p.recent); cudaFree(p.ring); cudaFree(p.cnt); cudaFree(p.drive_buf); cudaFree(p.stats);
            for (int c = 0; c < p.n_chan; ++c) { cudaFree(p.chan_in[c]); cudaFree(p.chan_s[c]); cudaFree(p.chan_r[c]); }
            cudaFree(p.flags);
        }
        for (auto& q : projs) {
            free_csr(q.csr);
            cudaFree(q.x_pre);
            cudaFree(q.x_post);
            cudaFree(q.seg_last); cudaFree(q.seg_x);
            cudaFree(q.pre_snap); cudaFree(q.post_ring); cudaFree(q.work_ctr);
        }
        cudaFree(d_step); cudaFree(d_events); cudaFree(d_raster_count); cudaFree(d_err);
        cudaFree(raster_step); cudaFree(raster_gid);
        sort_scratch.release();
        cudaFree(send); cudaFree(recv);
        if (comm) comm_destroy(&comm, comm_timeout_s);
        if (fork_ev) cudaEventDestroy(fork_ev);
        if (join_ev) cudaEventDestroy(join_ev);
        if (side) cudaStreamDestroy(side);
        if (stream) cudaStreamDestroy(stream);
    }

    float* acc_of(const EngineProj& q) const {
        const EnginePop& t = pops[q.tgt_pop];
        if (q.receptor >= NRN_RECV_CHANNEL) return t.chan_in[q.receptor - NRN_RECV_CHANNEL];
        return q.receptor == NRN_RECV_CURRENT ? t.d.i_syn : q.receptor == NRN_RECV_GEXC ? t.gin_exc : t.gin_inh;
    }

    nrn_proj_t dev_proj(const EngineProj& q) const {
        nrn_proj_t p{};
        p.n_src = q.csr.n_src;
        p.n_tgt = q.csr.n_tgt;
        p.dmin = q.csr.dmin;
        p.nd = q.csr.nd;
        p.src_hist = q.src_pop;
        p.max_seg = q.csr.max_seg;
        p.seg_ptr = q.csr.seg_ptr;
        p.tgt = q.csr.tgt;
        p.w = q.csr.w;
        p.mod = q.csr.mod;
        p.acc = acc_of(q);
        return p;
    }

    nrn_spike_hist_t hist(int i) const {
        nrn_spike_hist_t h{};
        h.ids = pops[i].hist_ids;
        h.count = pops[i].hist_count;
        h.cap = pops[i].hist_cap > 0 ? pops[i].hist_cap : 1;
        h.depth = depth;
        return h;
    }

    bool window_end(int64_t abs_step) const { return windows && (abs_step + 1) % win == 0; }

    nrn_pop_step_t pop_args(int i, double dt_step, int64_t step_off, bool in_run) const {
        const EnginePop& p = pops[i];
        nrn_pop_step_t a{};
        a.model = p.d.model;
        a.n = p.d.n;
        a.gid_offset = p.d.gid_offset + p.lo;
        a.dt = dt_step;
        a.v = p.d.v;
        a.aux = p.d.aux;
        a.refractory = p.d.refractory;
        a.spike = p.d.spike;
        a.i_syn = p.d.i_syn;
        if (p.cond) {
            a.g_exc = p.g_exc; a.g_inh = p.g_inh; a.gin_exc = p.gin_exc; a.gin_inh = p.gin_inh;
            a.tau_syn_exc = p.d.tau_syn_exc; a.tau_syn_inh = p.d.tau_syn_inh;
            a.e_exc = p.d.e_exc; a.e_inh = p.d.e_inh;
        }
        for (int k = 0; k < NRN_MAX_PARAMS; ++k) {
            a.param[k] = p.d.param[k];
            a.uniform[k] = p.d.uniform[k];
        }
        if (in_run) {
            a.n_chan = p.n_chan;
            for (int c = 0; c < p.n_chan; ++c) {
                a.chan_kind[c] = p.chan[c].kind;
                a.chan_tau_rise[c] = p.chan[c].tau_rise;
                a.chan_tau_decay[c] = p.chan[c].tau_decay;
                a.chan_e_rev[c] = static_cast<float>(p.chan[c].e_rev);
                a.chan_in[c] = p.chan_in[c];
                a.chan_s[c] = p.chan_s[c];
                a.chan_r[c] = p.chan_r[c];
            }
            a.drive = p.d.drive;
            a.step = step_off;
            a.step_base = reinterpret_cast<const int64_t*>(d_step);
            a.id_offset = p.lo;
            a.err = d_err;
            a.drive_values = p.drive_buf;
            a.spike_stats = p.stats;
            if (world > 1) {
                // ids go to the window send buffer; the ring is filled by the exchange
                a.win = win;
                a.send_hdr = send + p.send_off;
                a.send_ids = send + p.send_off + win + 1;
                a.send_cap = p.send_cap;
            } else {
                a.spike_ids = p.hist_ids;
                a.spike_count = p.hist_count;
                a.hist_depth = depth;
                a.hist_cap = p.hist_cap;
            }
            if (p.mask) {
                a.win = win;
                a.win_mask = p.mask + p.lo;
            }
            if (p.d.record) {
                a.raster_step = raster_step;
                a.raster_gid = raster_gid;
                a.raster_count = d_raster_count;
                a.raster_cap = raster_cap;
            }
            // traces of the plastic projections updated at every step
            a.trace_slow_ratio = slow_ratio;
            for (const auto& q : projs) {
                if (q.walk && q.tgt_pop == i) {
                    a.trace_ring[a.n_traces] = q.post_ring;
                    a.trace_ring_depth = ring_depth;
                    a.trace_decay[a.n_traces++] = static_cast<float>(std::exp(-dt / q.stdp[1]));
                }
                if (!q.plastic || !q.traces_fused) continue;
                if (q.src_pop == i) {
                    a.trace[a.n_traces] = q.x_pre;
                    a.trace_decay[a.n_traces++] = static_cast<float>(std::exp(-dt / q.stdp[0]));
                }
                if (q.tgt_pop == i) {
                    a.trace[a.n_traces] = q.x_post;
                    a.trace_decay[a.n_traces++] = static_cast<float>(std::exp(-dt / q.stdp[1]));
                }
            }
            if (p.recent) {
                a.post_recent = p.recent + static_cast<int64_t>(p.lo) * 4;
                a.post_ring = p.ring;
                a.post_cnt = p.cnt;
                a.post_ring_k = kRing;
            }
        }
        return a;
    }

    nrn_stdp_t stdp_args(const EngineProj& q) const {
        nrn_stdp_t s{};
        s.proj = dev_proj(q);
        s.w_mut = q.csr.w;
        s.in_ptr = q.csr.in_ptr;
        s.in_syn = q.csr.in_syn;
        s.in_src = q.csr.in_src;
        s.max_in = q.csr.max_in;
        s.max_row = q.csr.max_row;
        s.x_pre = q.x_pre;
        s.x_post = q.x_post;
        s.spike_src = pops[q.src_pop].d.spike;
        s.spike_tgt = pops[q.tgt_pop].d.spike;
        s.hist_src = hist(q.src_pop);
        s.hist_tgt = hist(q.tgt_pop);
        s.decay_pre = static_cast<float>(std::exp(-dt / q.stdp[0]));
        s.decay_post = static_cast<float>(std::exp(-dt / q.stdp[1]));
        s.a_plus = static_cast<float>(q.stdp[2]);
        s.a_minus = static_cast<float>(std::fabs(q.stdp[3]));
        s.w_min = static_cast<float>(q.stdp[4]);
        s.w_max = static_cast<float>(q.stdp[5]);
        s.lr = static_cast<float>(q.stdp[6]);
        s.slow_ratio = slow_ratio;
        s.traces_updated = q.traces_fused ? 1 : 0;
        return s;
    }

    WalkArgs walk_args(const EngineProj& q) const {
        const EnginePop& ps = pops[q.src_pop];
        const EnginePop& pt = pops[q.tgt_pop];
        WalkArgs a;
        a.n_src = q.csr.n_src;
        a.nd = q.csr.nd;
        a.dmin = q.csr.dmin;
        a.max_seg = q.csr.max_seg;
        a.seg_ptr = q.csr.seg_ptr;
        a.tgt = q.csr.tgt;
        a.w = q.csr.w;
        a.mod = q.csr.mod;
        a.acc = acc_of(q);
        a.hist_src = hist(q.src_pop);
        a.seg_last = q.seg_last;
        a.seg_x = q.seg_x;
        a.src_recent = reinterpret_cast<const int4*>(ps.recent);
        a.src_ring = ps.ring;
        a.src_cnt = ps.cnt;
        a.src_lo = ps.lo;
        a.src_hi = ps.lo + ps.d.n;
        a.tgt_recent = reinterpret_cast<const int4*>(pt.recent + static_cast<int64_t>(pt.lo) * 4);
        a.tgt_ring = pt.ring;
        a.tgt_cnt = pt.cnt;
        a.ring_k = kRing;
        a.pre_snap = q.pre_snap;
        a.pre_depth = q.pre_depth;
        a.post_ring = q.post_ring;
        a.post_depth = ring_depth;
        a.n_tgt = q.csr.n_tgt;
        a.win = win;
        a.decay_pre = static_cast<float>(std::exp(-dt / q.stdp[0]));
        a.decay_post = static_cast<float>(std::exp(-dt / q.stdp[1]));
        a.a_plus = static_cast<float>(q.stdp[2]);
        a.a_minus = static_cast<float>(std::fabs(q.stdp[3]));
        a.lr = static_cast<float>(q.stdp[6]);
        a.w_min = static_cast<float>(q.stdp[4]);
        a.w_max = static_cast<float>(q.stdp[5]);
        a.sweep_period = kSweepPeriod;
        a.sweep_rows = (q.csr.n_src + kSweepPeriod - 1) / kSweepPeriod;
        a.stale = kStale;
        a.err = d_err;
        a.events = d_events + 1;   // [1]: events delivered by the walks
        a.work_ctr = q.work_ctr;
        a.no_deliver = det ? 1 : 0;
        return a;
    }

    WindowArgs window_args(int i) const {
        const EnginePop& p = pops[i];
        WindowArgs a;
        a.n = p.n_global;
        a.mask = p.mask;
        a.win = win;
        a.err = d_err;
        a.own_lo = p.lo;
        a.own_hi = p.lo + p.d.n;
        for (const auto& q : projs) {
            if (!q.walk) continue;
            if (q.src_pop == i && a.n_task < 4) {
                SnapTask& t = a.task[a.n_task++];
                t.snap = q.pre_snap;
                t.depth = q.pre_depth;
                t.lo = 0;
                t.hi = p.n_global;
                t.decay = static_cast<float>(std::exp(-dt / q.stdp[0]));
                a.recent = reinterpret_cast<int4*>(p.recent);
                a.seg_last = q.seg_last;
                a.seg_nd = q.csr.nd;
            }
        }
        return a;
    }

    // Applies every pending update of the walk projections (weights are then
    // those after the last step run).
    nrn_status_t flush_walks() {
        if (step <= 0) return NRN_OK;
        for (auto& q : projs) {
            if (!q.walk) continue;
            if (world > 1 && step % win != 0)
                return fail(NRN_ERR_STATE, "partitioned network: read plastic weights at a window boundary (step " +
                                               std::to_string(step) + ", window " + std::to_string(win) + ")");
            NRN_TRY(walk_launch(walk_args(q), WALK_FLUSH, step, nullptr, stream));
        }
        return NRN_OK;
    }

    // Waits for the engine stream.  A partitioned engine polls it with the
    // communicator's time limit: a peer that stopped turns into NRN_ERR_COMM
    // (communicator aborted) instead of a hang.
    nrn_status_t wait_stream() {
        if (stuck) return fail(NRN_ERR_COMM, "the engine stream did not drain after the communicator was aborted");
        if (world > 1 && comm != nullptr) {
            const nrn_status_t st = comm_wait_stream(&comm, stream, comm_timeout_s, &stuck);
            if (st != NRN_OK) comm_failed = true;
            return st;
        }
        NRN_CUDA_TRY(cudaStreamSynchronize(stream));
        return NRN_OK;
    }

    nrn_status_t check_err() {
        int h = 0;
        NRN_CUDA_TRY(cudaMemcpyAsync(&h, d_err, sizeof(int), cudaMemcpyDeviceToHost, stream));
        NRN_TRY(wait_stream());
        if (h == 1) return fail(NRN_ERR_CAPACITY, "STDP: a neuron spiked more often than its spike history holds");
        if (h == 2) return fail(NRN_ERR_STATE, "STDP: a segment was not walked within the trace snapshot window");
        if (h == 3)
            return fail(NRN_ERR_STATE,
                        "STDP: a source on another GPU spiked twice within one synaptic delay; the partitioned "
                        "engine needs inter-spike intervals of plastic sources longer than their delays");
        if (h == 4)
            return fail(NRN_ERR_CAPACITY, "spike exchange buffer overflowed: raise max_rate_hz of the partition");
        return NRN_OK;
    }

    // Decides how each plastic projection is updated: by segment walks
    // (STDP at every step, at most 256 delays, one per source population),
    // else by the per-step kernels with the traces advanced in the neuron
    // updates where trace slots are free.
    void assign_plasticity() {
        std::vector<char> walk_src(pops.size(), 0);
        std::vector<int> used(pops.size(), 0);
        const char* eager = std::getenv("NRN_STDP_EAGER");   // per-step STDP kernels only (comparisons)
        const bool no_walk = eager && eager[0] == '1' && world == 1;
        for (auto& q : projs) {
            q.walk = false;
            if (no_walk || !q.plastic || slow_ratio != 1 || q.csr.nd > 256 || walk_src[q.src_pop] ||
                used[q.tgt_pop] >= NRN_MAX_TRACES)
                continue;
            walk_src[q.src_pop] = 1;
            used[q.tgt_pop] += 1;   // the target trace ring
            q.walk = true;
        }
        for (auto& q : projs) {
            q.traces_fused = false;
            if (!q.plastic || q.walk) continue;
            if (q.src_pop == q.tgt_pop) {
                if (used[q.src_pop] + 2 <= NRN_MAX_TRACES) {
                    used[q.src_pop] += 2;
                    q.traces_fused = true;
                }
            } else if (used[q.src_pop] < NRN_MAX_TRACES && used[q.tgt_pop] < NRN_MAX_TRACES) {
                used[q.src_pop] += 1;
                used[q.tgt_pop] += 1;
                q.traces_fused = true;
            }
        }
    }

    // Window end (after the last step's updates): spike exchange, then trace
    // snapshots.
    nrn_status_t enqueue_window_end(int64_t off) {
        if (world > 1) {
            if (comm == nullptr) return fail(NRN_ERR_STATE, "partitioned engine: the communicator was aborted");
            const ncclResult_t r =
                ncclAllGather(send, recv, static_cast<size_t>(rank_block), ncclInt32, comm, stream);
            if (r != ncclSuccess) {
                comm_failed = true;
                return comm_settle(&comm, r, comm_timeout_s, "ncclAllGather (window spike exchange)");
            }
            for (size_t i = 0; i < pops.size(); ++i) {
                const EnginePop& p = pops[i];
                UnpackArgs u;
                u.recv = recv;
                u.rank_stride = rank_block;
                u.pop_off = p.send_off;
                u.cap = p.send_cap;
                u.world = world;
                u.rank = rank;
                u.win = win;
                u.hist = hist(static_cast<int>(i));
                u.mask = p.mask;
                u.err = d_err;
                NRN_TRY(unpack_launch(u, off, d_step, stream));
            }
            for (const auto& p : pops)
                NRN_CUDA_TRY(cudaMemsetAsync(send + p.send_off, 0, static_cast<size_t>(win + 1) * sizeof(int32_t), stream));
        }
        for (size_t i = 0; i < pops.size(); ++i)
            if (pops[i].mask) NRN_TRY(window_launch(window_args(static_cast<int>(i)), off, d_step, stream));
        return NRN_OK;
    }

    // Enqueues one step at offset `off` from *d_step; with `ev` non-null,
    // records events around the three phases (ev[0..3]).  With `kev`
    // non-null every kernel runs on the main stream, one after the other,
    // with events between them (kev[0..6]: start, drive, static delivery,
    // STDP walks, neuron updates, per-step STDP, window end), for per-kernel
    // timing.
    nrn_status_t enqueue_step(int64_t off, bool win_end, cudaEvent_t* ev = nullptr, cudaEvent_t* kev = nullptr) {
        std::vector<nrn_proj_t> dp;
        for (auto& q : projs)
            if (!q.walk && !det) dp.push_back(dev_proj(q));
        std::vector<nrn_spike_hist_t> hs;
        for (size_t i = 0; i < pops.size(); ++i) hs.push_back(hist(static_cast<int>(i)));
        if (ev) NRN_CUDA_TRY(cudaEventRecord(ev[0], stream));
        if (kev) NRN_CUDA_TRY(cudaEventRecord(kev[0], stream));
        bool any_walk = false;
        for (auto& q : projs) any_walk = any_walk || q.walk;
        // Side stream, concurrent with the main stream's delivery work: this
        // step's external drive for every population (drawn ahead for the
        // neuron updates) and, with STDP walks on the main stream, the static
        // delivery (it also clears this step's history slots; the two touch
        // different history slots and only add into the accumulators).
        cudaStream_t sd = kev ? stream : side;
        if (!kev) {
            NRN_CUDA_TRY(cudaEventRecord(fork_ev, stream));
            NRN_CUDA_TRY(cudaStreamWaitEvent(side, fork_ev, 0));
        }
        {
            std::vector<nrn_pop_step_t> da;
            std::vector<float*> dout;
            for (size_t i = 0; i < pops.size(); ++i) {
                if (!pops[i].drive_buf) continue;
                da.push_back(pop_args(static_cast<int>(i), dt, off, true));
                dout.push_back(pops[i].drive_buf);
            }
            if (!da.empty()) NRN_TRY(drive_fill_group(da.data(), dout.data(), static_cast<int>(da.size()), sd));
        }
        if (kev) NRN_CUDA_TRY(cudaEventRecord(kev[1], stream));
        cudaStream_t ds = any_walk ? sd : stream;
        NRN_TRY(nrn_cuda_deliver_counted(dp.data(), static_cast<int32_t>(dp.size()), hs.data(),
                                         static_cast<int32_t>(hs.size()), off,
                                         reinterpret_cast<const int64_t*>(d_step), d_events,
                                         reinterpret_cast<nrn_stream_t>(ds)));
        if (kev) NRN_CUDA_TRY(cudaEventRecord(kev[2], stream));
        for (auto& q : projs)
            if (q.walk) NRN_TRY(walk_launch(walk_args(q), WALK_STEP, off, d_step, stream));
        if (kev) NRN_CUDA_TRY(cudaEventRecord(kev[3], stream));
        if (!kev) {
            NRN_CUDA_TRY(cudaEventRecord(join_ev, side));
            NRN_CUDA_TRY(cudaStreamWaitEvent(stream, join_ev, 0));
        }
        if (det) NRN_TRY(enqueue_det_delivery(off));
        if (ev) NRN_CUDA_TRY(cudaEventRecord(ev[1], stream));
        std::vector<nrn_pop_step_t> pa;
        for (size_t i = 0; i < pops.size(); ++i) pa.push_back(pop_args(static_cast<int>(i), dt, off, true));
        NRN_TRY(pop_step_group(pa.data(), static_cast<int>(pa.size()), stream));
        if (det)
            for (auto& p : pops)
                NRN_TRY(det_flags(p.d.spike, p.d.n, p.flags, det_ring, off, d_step, stream));
        for (const auto& pr : probes) {
            const EnginePop& p = pops[pr.pop];
            const float* src = pr.var == NRN_VAR_V ? p.d.v : pr.var == NRN_VAR_AUX ? p.d.aux
                             : pr.var == NRN_VAR_REFRACTORY ? p.d.refractory : pr.var == NRN_VAR_SPIKE ? p.d.spike
                             : p.d.i_syn;
            const int blocks = std::max(1, std::min((p.d.n + 255) / 256, 4 * sm_count_current()));
            probe_kernel<<<blocks, 256, 0, stream>>>(src, p.d.n, pr.ring, pr.depth, off, d_step);
            NRN_CUDA_TRY(cudaGetLastError());
        }
        if (ev) NRN_CUDA_TRY(cudaEventRecord(ev[2], stream));
        if (kev) NRN_CUDA_TRY(cudaEventRecord(kev[4], stream));
        for (auto& q : projs) {
            if (!q.plastic || q.walk) continue;
            nrn_stdp_t s = stdp_args(q);
            NRN_TRY(nrn_cuda_stdp_step(&s, off, reinterpret_cast<const int64_t*>(d_step),
                                        reinterpret_cast<nrn_stream_t>(stream)));
        }
        if (kev) NRN_CUDA_TRY(cudaEventRecord(kev[5], stream));
        if (win_end) NRN_TRY(enqueue_window_end(off));
        if (ev) NRN_CUDA_TRY(cudaEventRecord(ev[3], stream));
        if (kev) NRN_CUDA_TRY(cudaEventRecord(kev[6], stream));
        return NRN_OK;
    }

    // Deterministic delivery of this step into every input of every
    // population (projections in index order), after the walks updated the
    // weights of the arriving spikes' segments.
    nrn_status_t enqueue_det_delivery(int64_t off) {
        for (size_t i = 0; i < pops.size(); ++i) {
            const EnginePop& t = pops[i];
            const int n_acc = 3 + t.n_chan;
            for (int r = 0; r < n_acc; ++r) {
                const int receptor = r < 3 ? r : NRN_RECV_CHANNEL + (r - 3);
                DetAcc A;
                A.n = t.d.n;
                for (const auto& q : projs) {
                    if (q.tgt_pop != static_cast<int>(i) || q.receptor != receptor) continue;
                    if (A.nproj == 8) return fail(NRN_ERR_UNSUPPORTED, "deterministic delivery: more than 8 "
                                                                      "projections into one input");
                    DetProj& P = A.proj[A.nproj++];
                    P.ptr = q.csr.det_ptr;
                    P.syn = q.csr.det_syn;
                    P.src = q.csr.det_src;
                    P.delay = q.csr.det_delay;
                    P.w = q.csr.w;
                    P.mod = q.csr.mod;
                    P.flags = pops[q.src_pop].flags;
                    P.flag_n = pops[q.src_pop].n_global;
                    A.acc = acc_of(q);
                }
                if (A.nproj == 0) continue;
                NRN_TRY(det_deliver(A, det_ring, off, d_step, d_events, stream));
            }
        }
        return NRN_OK;
    }

    // A graph of `chunk` steps starting at a window start (when windows are on).
    // Graph length of whole-window pieces (0 picks 50 steps, rounded to windows).
    int run_chunk(int chunk) const {
        if (chunk <= 0) chunk = 50;
        const int w = windows ? win : 1;
        return windows ? std::max(w, chunk / w * w) : chunk;
    }
    // The length of the next graph of a run that is at window phase `phase`
    // with `left` steps to go.
    int run_piece(int phase, int64_t left, int chunk) const {
        const int w = windows ? win : 1;
        if (phase != 0) return 1;
        if (left >= w && w > 1) return static_cast<int>(std::min<int64_t>(chunk, left / w * w));
        if (w > 1) return static_cast<int>(left);   // a tail shorter than a window: one graph
        if (left >= chunk) return chunk;
        int c = 1;
        while (2 * c <= left) c *= 2;
        return c;
    }

    nrn_status_t graph_for(int chunk, cudaGraphExec_t* out, int phase = 0) {
        const auto key = std::make_pair(phase, chunk);
        auto it = graphs.find(key);
        if (it != graphs.end()) {
            *out = it->second;
            return NRN_OK;
        }
        cudaGraph_t g = nullptr;
        NRN_CUDA_TRY(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
        nrn_status_t st = NRN_OK;
        for (int k = 0; k < chunk && st == NRN_OK; ++k) st = enqueue_step(k, window_end(phase + k));
        if (st == NRN_OK) {
            advance_kernel<<<1, 1, 0, stream>>>(d_step, chunk);
            if (cudaGetLastError() != cudaSuccess) st = fail(NRN_ERR_CUDA, "advance_kernel launch failed");
        }
        cudaError_t e = cudaStreamEndCapture(stream, &g);
        if (st != NRN_OK) {
            if (g) cudaGraphDestroy(g);
            return st;
        }
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
        cudaGraphExec_t ex = nullptr;
        e = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
        // the upload a first launch would do, done now (ahead of a timed run)
        e = cudaGraphUpload(ex, stream);
        if (e != cudaSuccess) {
            cudaGraphExecDestroy(ex);
            return cuda_fail(e, "cudaGraphUpload");
        }
        graphs[key] = ex;
        *out = ex;
        return NRN_OK;
    }

    // One step launched directly (absolute step `abs`, = *d_step).
    nrn_status_t eager_step(int64_t abs) {
        NRN_TRY(enqueue_step(0, window_end(abs)));
        advance_kernel<<<1, 1, 0, stream>>>(d_step, 1);
        NRN_CUDA_TRY(cudaGetLastError());
        return NRN_OK;
    }

    // The walk launches' unit counters start at zero (the launch of step s
    // uses counter s % 2 and clears the other for step s + 1; a run may start
    // at any step).
    nrn_status_t reset_walk_ctr() {
        for (auto& q : projs)
            if (q.work_ctr) NRN_CUDA_TRY(cudaMemsetAsync(q.work_ctr, 0, 3 * sizeof(unsigned int), stream));
        return NRN_OK;
    }

    // First run: weights clamped, walk state starting at the current step.
    nrn_status_t prepare_plastic() {
        NRN_TRY(reset_walk_ctr());
        for (auto& q : projs) {
            if (!q.plastic || q.clamped) continue;
            // The reference clamps every weight of a plastic connection on
            // each update (stdp.cpp:139); one clamp of all weights before the
            // first update, then of each changed weight, is the same.
            NRN_TRY(nrn_cuda_clamp(q.csr.w, q.csr.nnz, static_cast<float>(q.stdp[4]), static_cast<float>(q.stdp[5]),
                                   reinterpret_cast<nrn_stream_t>(stream)));
            if (q.walk) {
                const std::vector<int32_t> last(static_cast<size_t>(q.csr.n_src) * q.csr.nd,
                                                static_cast<int32_t>(step - 1));
                NRN_CUDA_TRY(cudaMemcpyAsync(q.seg_last, last.data(), last.size() * sizeof(int32_t),
                                             cudaMemcpyHostToDevice, stream));
                NRN_TRY(wait_stream());
            }
            q.clamped = true;
        }
        return NRN_OK;
    }

    void drop_graphs() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        graphs.clear();
    }

    // Every device buffer a checkpoint holds, in a fixed order (buffers an
    // engine does not have are left out; an engine built from the same
    // network has the same list).
    struct StateBuf {
        void* p;
        size_t bytes;
    };
    std::vector<StateBuf> state_buffers() {
        std::vector<StateBuf> b;
        auto add = [&](void* p, size_t bytes) {
            if (p != nullptr && bytes > 0) b.push_back({p, bytes});
        };
        for (auto& p : pops) {
            const size_t n = static_cast<size_t>(p.d.n);
            add(p.d.v, n * 4);
            add(p.d.aux, n * 4);
            add(p.d.refractory, n * 4);
            add(p.d.spike, n * 4);
            add(p.d.i_syn, n * 4);
            add(p.g_exc, n * 4);
            add(p.g_inh, n * 4);
            add(p.gin_exc, n * 4);
            add(p.gin_inh, n * 4);
            add(p.hist_ids, static_cast<size_t>(depth) * p.hist_cap * 4);
            add(p.hist_count, static_cast<size_t>(depth) * 4);
            add(p.mask, static_cast<size_t>(p.n_global) * 4);
            add(p.recent, static_cast<size_t>(p.n_global) * 16);
            add(p.ring, n * kRing * 4);
            add(p.cnt, n * 4);
            add(p.stats, n * sizeof(nrn_spike_stat_t));
            add(p.flags, static_cast<size_t>(det_ring) * p.n_global);
            for (int c = 0; c < p.n_chan; ++c) {
                add(p.chan_in[c], n * 4);
                add(p.chan_s[c], n * 4);
                add(p.chan_r[c], n * 4);
            }
        }
        for (auto& q : projs) {
            add(q.csr.w, static_cast<size_t>(q.csr.nnz) * 4);
            add(q.x_pre, static_cast<size_t>(pops[q.src_pop].d.n) * 4);
            add(q.x_post, static_cast<size_t>(pops[q.tgt_pop].d.n) * 4);
            if (q.walk) {
                const size_t nseg = static_cast<size_t>(q.csr.n_src) * q.csr.nd;
                add(q.seg_last, nseg * 4);
                add(q.seg_x, nseg * 4);
                add(q.pre_snap, static_cast<size_t>(q.pre_depth) * q.csr.n_src * 4);
                add(q.post_ring, static_cast<size_t>(ring_depth) * q.csr.n_tgt * 4);
            }
        }
        add(d_events, 2 * sizeof(unsigned long long));
        return b;
    }
};

// Checkpoint layout: header, the byte count of every state buffer, one
// flag byte per projection (weights already clamped), padded to 8 bytes,
// the buffers, then the raster not yet read (steps, then ids).
struct CkptHeader {
    char magic[8];
    int64_t step;
    int64_t spikes_flushed;
    int64_t raster_n;
    int32_t world, rank;
    int32_t n_buf, n_proj;
};
constexpr char kCkptMagic[8] = {'N', 'R', 'N', 'C', 'K', 'P', 'T', '1'};

#define ENGINE_GUARD(e)                                                          \
    do {                                                                         \
        if ((e) == nullptr) return fail(NRN_ERR_INVALID, "null engine");         \
        cudaError_t ce_ = cudaSetDevice((e)->device);                            \
        if (ce_ != cudaSuccess) return cuda_fail(ce_, "cudaSetDevice");          \
    } while (0)

namespace nrn {

nrn_status_t engine_raster_view(nrn_engine* e, EngineRasterView* v) {
    NRN_CHECK_ARG(e != nullptr && v != nullptr, "null engine");
    if (!e->finalized) return fail(NRN_ERR_STATE, "raster read before nrn_engine_finalize");
    v->device = e->device;
    v->stream = e->stream;
    v->step = e->raster_step;
    v->gid = e->raster_gid;
    v->count = e->d_raster_count;
    v->cap = e->raster_cap;
    v->flushed = &e->spikes_flushed;
    return NRN_OK;
}

}  // namespace nrn

extern "C" {

const char* nrn_status_string(nrn_status_t s) {
    switch (s) {
        case NRN_OK: return "ok";
        case NRN_ERR_INVALID: return "invalid argument";
        case NRN_ERR_CUDA: return "CUDA error";
        case NRN_ERR_OOM: return "out of device memory";
        case NRN_ERR_CAPACITY: return "buffer capacity exceeded";
        case NRN_ERR_UNSUPPORTED: return "unsupported device";
        case NRN_ERR_COMM: return "collective communication error";
        case NRN_ERR_TIMEOUT: return "device wait timed out";
        case NRN_ERR_STATE: return "call out of order";
    }
    return "unknown status";
}

const char* nrn_last_error(void) { return nrn::g_last_error.c_str(); }

const char* nrn_version(void) { return "0.1.0 sm_100a"; }

nrn_status_t nrn_engine_create(nrn_engine** out, int device, double dt, int32_t slow_ratio) {
    NRN_CHECK_ARG(out != nullptr, "nrn_engine_create: null output");
    NRN_CHECK_ARG(dt > 0.0, "nrn_engine_create: dt must be positive");
    NRN_CHECK_ARG(slow_ratio >= 1, "nrn_engine_create: slow_ratio must be >= 1");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(NRN_ERR_UNSUPPORTED, "no CUDA device");
    }
    NRN_CHECK_ARG(device >= 0 && device < ndev, "nrn_engine_create: bad device index");
    NRN_CUDA_TRY(cudaSetDevice(device));
    cudaDeviceProp prop{};
    NRN_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return fail(NRN_ERR_UNSUPPORTED, std::string("libnrn_b200 is built for sm_100a; device is ") + prop.name);
    auto e = std::make_unique<nrn_engine>();
    e->device = device;
    e->dt = dt;
    e->slow_ratio = slow_ratio;
    const char* ng = std::getenv("NRN_NO_GRAPHS");
    e->use_graphs = !(ng && ng[0] == '1');
    NRN_CUDA_TRY(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    NRN_CUDA_TRY(cudaStreamCreateWithFlags(&e->side, cudaStreamNonBlocking));
    NRN_CUDA_TRY(cudaEventCreateWithFlags(&e->fork_ev, cudaEventDisableTiming));
    NRN_CUDA_TRY(cudaEventCreateWithFlags(&e->join_ev, cudaEventDisableTiming));
    NRN_TRY(dalloc0(&e->d_step, 1, e->stream));
    NRN_TRY(dalloc0(&e->d_events, 2, e->stream));   // [0] static delivery, [1] walks
    NRN_TRY(dalloc0(&e->d_raster_count, 1, e->stream));
    NRN_TRY(dalloc0(&e->d_err, 1, e->stream));
    *out = e.release();
    return NRN_OK;
}

nrn_status_t nrn_engine_destroy(nrn_engine* e) {
    if (e == nullptr) return NRN_OK;
    cudaSetDevice(e->device);
    e->wait_stream();
    delete e;
    return NRN_OK;
}

nrn_status_t nrn_comm_unique_id(uint8_t id[128]) {
    NRN_CHECK_ARG(id != nullptr, "nrn_comm_unique_id: null output");
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");
    ncclUniqueId u;
    ncclResult_t r = ncclGetUniqueId(&u);
    if (r != ncclSuccess) return fail(NRN_ERR_COMM, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
    std::memcpy(id, &u, sizeof(u));
    return NRN_OK;
}

nrn_status_t nrn_engine_set_partition(nrn_engine* e, int32_t rank, int32_t world, const uint8_t id[128],
                                      double max_rate_hz) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(e->pops.empty() && !e->finalized, "nrn_engine_set_partition: call before adding populations");
    NRN_CHECK_ARG(world >= 1 && rank >= 0 && rank < world, "nrn_engine_set_partition: bad rank or world size");
    NRN_CHECK_ARG(max_rate_hz > 0.0, "nrn_engine_set_partition: max_rate_hz must be positive");
    NRN_CHECK_ARG(e->comm == nullptr, "nrn_engine_set_partition: already partitioned");
    e->max_rate_hz = max_rate_hz;
    e->rank = rank;
    e->world = world;
    if (world == 1) return NRN_OK;
    NRN_CHECK_ARG(id != nullptr, "nrn_engine_set_partition: null NCCL id");
    const nrn_status_t st = comm_init(&e->comm, world, id, rank, e->comm_timeout_s);
    if (st != NRN_OK) {
        e->comm = nullptr;
        e->world = 1;
        e->rank = 0;
        return st;
    }
    return NRN_OK;
}

nrn_status_t nrn_engine_stream(nrn_engine* e, nrn_stream_t* stream) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(stream != nullptr, "null output");
    *stream = reinterpret_cast<nrn_stream_t>(e->stream);
    return NRN_OK;
}

int64_t nrn_engine_step(const nrn_engine* e) { return e ? e->step : -1; }

nrn_status_t nrn_engine_info(const nrn_engine* e, nrn_engine_info_t* out) {
    NRN_CHECK_ARG(e != nullptr && out != nullptr, "nrn_engine_info: null argument");
    NRN_CHECK_ARG(e->finalized, "nrn_engine_info: finalize first");
    out->window = e->windows ? e->win : 1;
    out->n_pops = static_cast<int32_t>(e->pops.size());
    out->raster_capacity = e->raster_cap;
    int64_t rec = 0;
    for (const auto& p : e->pops)
        if (p.d.record) rec += p.d.n;
    out->recorded_neurons = rec;
    out->step = e->step;
    return NRN_OK;
}

nrn_status_t nrn_engine_add_population(nrn_engine* e, const nrn_pop_desc_t* d, int32_t* id) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(d != nullptr, "null population");
    NRN_CHECK_ARG(!e->finalized, "nrn_engine_add_population: engine already finalized");
    NRN_CHECK_ARG(e->pops.size() < NRN_MAX_POPS, "too many populations");
    NRN_CHECK_ARG(d->model >= NRN_MODEL_LIF && d->model <= NRN_MODEL_IZH, "unknown model");
    NRN_CHECK_ARG(d->n > 0, "population must have at least 1 neuron");
    NRN_CHECK_ARG(d->v && d->spike, "population needs v and spike arrays");
    NRN_CHECK_ARG(d->model == NRN_MODEL_LIF || d->aux, "population needs aux (w/u)");
    NRN_CHECK_ARG(d->model == NRN_MODEL_IZH || d->refractory, "population needs refractory");
    EnginePop p;
    p.d = *d;
    p.n_global = d->n_global > 0 ? d->n_global : d->n;
    p.lo = d->local_offset;
    NRN_CHECK_ARG(p.lo >= 0 && p.lo + d->n <= p.n_global, "population slice outside the population");
    NRN_CHECK_ARG(e->world > 1 || (p.lo == 0 && p.n_global == d->n),
                  "a population slice (n_global, local_offset) needs nrn_engine_set_partition");
    p.cond = d->tau_syn_exc > 0.0f;
    NRN_CHECK_ARG(!p.cond || d->model == NRN_MODEL_ADEX, "conductance input is supported for AdEx");
    NRN_CHECK_ARG(d->drive.kind != NRN_DRIVE_POISSON_GEXC || p.cond, "conductance drive needs conductance input");
    if (p.d.i_syn == nullptr) {
        NRN_TRY(dalloc0(&p.d.i_syn, static_cast<size_t>(d->n), e->stream));
        p.owns_isyn = true;
    }
    if (p.cond) {
        NRN_TRY(dalloc0(&p.g_exc, d->n, e->stream));
        NRN_TRY(dalloc0(&p.g_inh, d->n, e->stream));
        NRN_TRY(dalloc0(&p.gin_exc, d->n, e->stream));
        NRN_TRY(dalloc0(&p.gin_inh, d->n, e->stream));
    }
    e->pops.push_back(p);
    if (id) *id = static_cast<int32_t>(e->pops.size() - 1);
    return NRN_OK;
}

nrn_status_t nrn_engine_set_params(nrn_engine* e, int32_t pop, const float* const* param, const float* uniform) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(pop >= 0 && pop < static_cast<int32_t>(e->pops.size()), "bad population index");
    auto& d = e->pops[pop].d;
    bool changed = false;
    for (int k = 0; k < NRN_MAX_PARAMS; ++k) {
        const float* p = param ? param[k] : nullptr;
        const float u = uniform ? uniform[k] : d.uniform[k];
        changed = changed || p != d.param[k] || u != d.uniform[k];
        d.param[k] = p;
        d.uniform[k] = u;
    }
    if (changed) e->drop_graphs();
    return NRN_OK;
}

static nrn_status_t check_receptor(nrn_engine* e, int32_t tgt, int32_t receptor) {
    const EnginePop& t = e->pops[tgt];
    if (receptor >= NRN_RECV_CHANNEL) {
        NRN_CHECK_ARG(receptor - NRN_RECV_CHANNEL < t.n_chan, "receptor names a synapse channel the target lacks");
        return NRN_OK;
    }
    NRN_CHECK_ARG(receptor >= NRN_RECV_CURRENT && receptor <= NRN_RECV_GINH, "bad receptor");
    NRN_CHECK_ARG(receptor == NRN_RECV_CURRENT || t.cond,
                  "conductance receptor on a population without conductance input");
    return NRN_OK;
}

nrn_status_t nrn_engine_add_synapse_channel(nrn_engine* e, int32_t pop, const nrn_syn_desc_t* d, int32_t* channel) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(d != nullptr, "null synapse channel");
    NRN_CHECK_ARG(!e->finalized, "nrn_engine_add_synapse_channel: engine already finalized");
    NRN_CHECK_ARG(pop >= 0 && pop < static_cast<int32_t>(e->pops.size()), "bad population index");
    EnginePop& p = e->pops[pop];
    NRN_CHECK_ARG(p.n_chan < NRN_MAX_CHANNELS, "at most 4 synapse channels per population");
    NRN_CHECK_ARG(d->kind >= NRN_SYN_EXP && d->kind <= NRN_SYN_AMPA, "unknown synapse channel kind");
    NRN_CHECK_ARG(d->tau_decay > 0.0 && (d->kind == NRN_SYN_EXP || d->tau_rise > 0.0) && std::isfinite(d->e_rev),
                  "synapse time constants must be positive");
    const int c = p.n_chan;
    const size_t n = static_cast<size_t>(p.d.n);
    NRN_TRY(dalloc0(&p.chan_in[c], n, e->stream));
    NRN_TRY(dalloc0(&p.chan_s[c], n, e->stream));
    if (d->kind != NRN_SYN_EXP) NRN_TRY(dalloc0(&p.chan_r[c], n, e->stream));
    p.chan[c] = *d;
    p.n_chan = c + 1;
    e->drop_graphs();
    if (channel) *channel = c;
    return NRN_OK;
}

static nrn_status_t add_projection_dev(nrn_engine* e, int32_t src_pop, int32_t tgt_pop, int32_t receptor,
                                       const int32_t* src, const int32_t* tgt, const float* w, const uint8_t* delay,
                                       const float* mod, int64_t n, bool keep_orig, int32_t dmin, int32_t dmax,
                                       int32_t* id) {
    EngineProj q;
    q.src_pop = src_pop;
    q.tgt_pop = tgt_pop;
    q.receptor = receptor;
    q.csr.dmin = dmin;
    q.csr.nd = dmax - dmin + 1;
    NRN_TRY(build_csr(q.csr, e->pops[src_pop].n_global, e->pops[tgt_pop].d.n, src, tgt, w, delay, mod, n, keep_orig,
                      e->stream));
    e->projs.push_back(q);
    e->drop_graphs();
    if (id) *id = static_cast<int32_t>(e->projs.size() - 1);
    return NRN_OK;
}

nrn_status_t nrn_engine_add_projection(nrn_engine* e, const nrn_proj_desc_t* d, int32_t* id) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(d != nullptr, "null projection");
    NRN_CHECK_ARG(!e->finalized, "nrn_engine_add_projection: engine already finalized");
    NRN_CHECK_ARG(e->projs.size() < NRN_MAX_PROJ, "too many projections");
    const int np = static_cast<int>(e->pops.size());
    NRN_CHECK_ARG(d->src_pop >= 0 && d->src_pop < np && d->tgt_pop >= 0 && d->tgt_pop < np, "bad population index");
    NRN_TRY(check_receptor(e, d->tgt_pop, d->receptor));
    NRN_CHECK_ARG(d->nnz >= 0, "negative synapse count");
    NRN_CHECK_ARG(d->nnz == 0 || (d->src && d->tgt && d->w && d->delay), "null synapse arrays");
    const int64_t n = d->nnz;
    // delay range (scan on the host copy or after upload)
    std::vector<uint8_t> hd(static_cast<size_t>(n));
    if (n > 0) {
        if (d->on_device) NRN_CUDA_TRY(cudaMemcpy(hd.data(), d->delay, n, cudaMemcpyDeviceToHost));
        else std::memcpy(hd.data(), d->delay, n);
    }
    int dmin = 255, dmax = 1;
    for (uint8_t x : hd) {
        dmin = std::min<int>(dmin, x);
        dmax = std::max<int>(dmax, x);
    }
    if (n == 0) dmin = dmax = 1;
    NRN_CHECK_ARG(dmin >= 1, "synaptic delays must be >= 1 step");
    if (d->on_device)
        return add_projection_dev(e, d->src_pop, d->tgt_pop, d->receptor, d->src, d->tgt, d->w, d->delay, d->mod, n,
                                  true, dmin, dmax, id);
    int32_t *s = nullptr, *t = nullptr;
    float *w = nullptr, *m = nullptr;
    uint8_t* dl = nullptr;
    auto cleanup = [&]() { cudaFree(s); cudaFree(t); cudaFree(w); cudaFree(m); cudaFree(dl); };
    nrn_status_t st = NRN_OK;
    if ((st = dalloc0(&s, n, e->stream)) != NRN_OK || (st = dalloc0(&t, n, e->stream)) != NRN_OK ||
        (st = dalloc0(&w, n, e->stream)) != NRN_OK || (st = dalloc0(&dl, n, e->stream)) != NRN_OK ||
        (d->mod && (st = dalloc0(&m, n, e->stream)) != NRN_OK)) {
        cleanup();
        return st;
    }
    cudaError_t ce = cudaSuccess;
    if (n > 0) {
        ce = cudaMemcpyAsync(s, d->src, n * 4, cudaMemcpyHostToDevice, e->stream);
        if (ce == cudaSuccess) ce = cudaMemcpyAsync(t, d->tgt, n * 4, cudaMemcpyHostToDevice, e->stream);
        if (ce == cudaSuccess) ce = cudaMemcpyAsync(w, d->w, n * 4, cudaMemcpyHostToDevice, e->stream);
        if (ce == cudaSuccess) ce = cudaMemcpyAsync(dl, d->delay, n, cudaMemcpyHostToDevice, e->stream);
        if (ce == cudaSuccess && d->mod) ce = cudaMemcpyAsync(m, d->mod, n * 4, cudaMemcpyHostToDevice, e->stream);
    }
    if (ce != cudaSuccess) {
        cleanup();
        return cuda_fail(ce, "projection upload");
    }
    st = add_projection_dev(e, d->src_pop, d->tgt_pop, d->receptor, s, t, w, dl, m, n, true, dmin, dmax, id);
    e->wait_stream();
    cleanup();
    return st;
}

nrn_status_t nrn_engine_generate_projection(nrn_engine* e, const nrn_gen_desc_t* g, int32_t* id, int64_t* nnz) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(g != nullptr, "null generator");
    NRN_CHECK_ARG(!e->finalized, "engine already finalized");
    NRN_CHECK_ARG(e->projs.size() < NRN_MAX_PROJ, "too many projections");
    const int np = static_cast<int>(e->pops.size());
    NRN_CHECK_ARG(g->src_pop >= 0 && g->src_pop < np && g->tgt_pop >= 0 && g->tgt_pop < np, "bad population index");
    NRN_CHECK_ARG(g->degree >= 0 && g->dmin >= 1 && g->dmax >= g->dmin && g->dmax <= 255, "bad generator range");
    NRN_TRY(check_receptor(e, g->tgt_pop, g->receptor));
    const EnginePop& ps = e->pops[g->src_pop];
    const EnginePop& pt = e->pops[g->tgt_pop];
    if (g->rule == NRN_GEN_ER || g->rule == NRN_GEN_DISTANCE) {
        NRN_CHECK_ARG(g->rule != NRN_GEN_ER || (g->p >= 0.0 && g->p <= 1.0), "ER probability outside [0, 1]");
        NRN_CHECK_ARG(g->rule != NRN_GEN_DISTANCE ||
                          (g->sigma > 0.0 && g->max_distance > 0.0 && g->min_probability >= 0.0 &&
                           g->min_probability <= 1.0),
                      "distance rule: sigma and max_distance must be positive, min_probability in [0, 1]");
        RandArgs a;
        a.rule = g->rule;
        a.seed = g->seed;
        a.gen_id = static_cast<uint32_t>(g->gen_id);
        a.n_src = ps.n_global;
        a.n_tgt = pt.n_global;
        a.tgt_lo = pt.lo;
        a.n_rows = pt.d.n;
        a.tgt_gid_offset = pt.d.gid_offset;
        a.same_pop = g->src_pop == g->tgt_pop;
        a.p = g->p;
        a.log1mp = g->p < 1.0 ? det_log(1.0 - g->p) : 0.0;
        a.spacing_src = ps.n_global > 1 ? g->max_distance / ps.n_global : 0.0;
        a.spacing_tgt = pt.n_global > 1 ? g->max_distance / pt.n_global : 0.0;
        a.inv_two_sigma_sq = g->rule == NRN_GEN_DISTANCE ? 1.0 / (2.0 * g->sigma * g->sigma) : 0.0;
        a.p_min = g->min_probability;
        // beyond sigma * sqrt(2 ln 2^40) the Gaussian is below 2^-40: no pair
        // there can pass the 32-bit threshold
        a.half_window = g->min_probability > 0.0 ? -1.0 : g->sigma * std::sqrt(2.0 * 40.0 * kLn2);
        a.dmin = g->dmin;
        a.dmax = g->dmax;
        a.w_lo = g->w_lo;
        a.w_span = g->w_span;
        DevSynList list;
        NRN_TRY(generate_random(a, &list, e->stream));
        nrn_status_t st = add_projection_dev(e, g->src_pop, g->tgt_pop, g->receptor, list.src, list.tgt, list.w,
                                             list.delay, nullptr, list.n, false, g->dmin, g->dmax, id);
        e->wait_stream();
        list.release();
        if (st == NRN_OK && nnz) *nnz = e->projs.back().csr.nnz;
        return st;
    }
    NRN_CHECK_ARG(g->rule == NRN_GEN_FIXED, "unknown connectivity rule");
    // sources over the whole population, targets on this rank
    const int32_t src_gid = ps.d.gid_offset, tgt_gid = pt.d.gid_offset;
    GenArgs a{};
    a.out_degree = g->out_degree;
    a.degree = g->degree;
    a.gen_id = static_cast<uint32_t>(g->gen_id);
    a.n_src = ps.n_global;
    a.src_offset = src_gid;
    a.col_offset = g->col_n > 0 ? g->col_offset : (g->out_degree ? tgt_gid : src_gid);
    a.col_n = g->col_n > 0 ? g->col_n : (g->out_degree ? pt.n_global : ps.n_global);
    a.row_offset = g->out_degree ? src_gid : tgt_gid + pt.lo;
    a.n_rows = g->out_degree ? ps.n_global : pt.d.n;
    a.keep_lo = tgt_gid + pt.lo;
    a.keep_hi = tgt_gid + pt.lo + pt.d.n;
    a.dmin = g->dmin;
    a.dmax = g->dmax;
    a.w_lo = g->w_lo;
    a.w_span = g->w_span;
    a.seed = g->seed;
    const int64_t total = static_cast<int64_t>(a.n_rows) * a.degree;
    int32_t *s = nullptr, *t = nullptr;
    float* w = nullptr;
    uint8_t* dl = nullptr;
    auto cleanup = [&]() { cudaFree(s); cudaFree(t); cudaFree(w); cudaFree(dl); };
    nrn_status_t st = NRN_OK;
    if ((st = dalloc0(&s, total, e->stream)) != NRN_OK || (st = dalloc0(&t, total, e->stream)) != NRN_OK ||
        (st = dalloc0(&w, total, e->stream)) != NRN_OK || (st = dalloc0(&dl, total, e->stream)) != NRN_OK) {
        cleanup();
        return st;
    }
    st = generate(a, s, t, w, dl, e->stream);
    if (st == NRN_OK)
        st = add_projection_dev(e, g->src_pop, g->tgt_pop, g->receptor, s, t, w, dl, nullptr, total, false, g->dmin,
                                g->dmax, id);
    e->wait_stream();
    cleanup();
    if (st == NRN_OK && nnz) *nnz = e->projs.back().csr.nnz;
    return st;
}

nrn_status_t nrn_engine_set_stdp(nrn_engine* e, int32_t proj, const double* p) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(proj >= 0 && proj < static_cast<int32_t>(e->projs.size()), "bad projection index");
    NRN_CHECK_ARG(p != nullptr, "null STDP parameters");
    NRN_CHECK_ARG(p[0] > 0 && p[1] > 0, "STDP time constants must be positive");
    for (int k = 0; k < 7; ++k) NRN_CHECK_ARG(std::isfinite(p[k]), "STDP parameters must be finite");
    NRN_CHECK_ARG(p[4] <= p[5], "STDP needs w_min <= w_max");
    NRN_CHECK_ARG(!e->finalized, "nrn_engine_set_stdp: set plasticity before nrn_engine_finalize");
    auto& q = e->projs[proj];
    std::memcpy(q.stdp, p, sizeof(q.stdp));
    q.plastic = true;
    e->drop_graphs();
    return NRN_OK;
}

// Every rank of a partitioned network must agree on the exchange layout:
// the all-gather moves rank_block ids from each rank, and a rank whose count
// differs leaves the others waiting.  At finalize the ranks exchange a
// fixed-size record of what sets the layout (one all-gather of a fixed
// count, which cannot disagree) and compare it.
static nrn_status_t check_layout(nrn_engine* e) {
    constexpr int kRec = 128;
    std::vector<long long> rec(kRec, 0);
    auto bits = [](double x) {
        long long b = 0;
        std::memcpy(&b, &x, sizeof(b));
        return b;
    };
    rec[0] = 0x4E524E4C41594F55LL;   // record tag
    rec[1] = e->world;
    rec[2] = e->win;
    rec[3] = e->depth;
    rec[4] = e->rank_block;
    rec[5] = static_cast<long long>(e->pops.size());
    rec[6] = static_cast<long long>(e->projs.size());
    rec[7] = bits(e->dt);
    rec[8] = e->slow_ratio;
    rec[9] = bits(e->max_rate_hz);
    for (size_t i = 0; i < e->pops.size(); ++i) {
        rec[16 + i] = e->pops[i].send_cap;
        rec[16 + NRN_MAX_POPS + i] = e->pops[i].n_global;
        rec[16 + 2 * NRN_MAX_POPS + i] = e->pops[i].send_off;
    }
    long long* d = nullptr;
    NRN_TRY(dalloc0(&d, static_cast<size_t>(kRec) * (1 + e->world), e->stream));
    std::vector<long long> all(static_cast<size_t>(kRec) * e->world);
    nrn_status_t st = NRN_OK;
    cudaError_t ce = cudaMemcpyAsync(d, rec.data(), kRec * sizeof(long long), cudaMemcpyHostToDevice, e->stream);
    if (ce != cudaSuccess) st = cuda_fail(ce, "layout record upload");
    if (st == NRN_OK) {
        const ncclResult_t r = ncclAllGather(d, d + kRec, kRec, ncclInt64, e->comm, e->stream);
        st = comm_settle(&e->comm, r, e->comm_timeout_s, "ncclAllGather (exchange layout check)");
        if (st != NRN_OK) e->comm_failed = true;
    }
    if (st == NRN_OK) {
        ce = cudaMemcpyAsync(all.data(), d + kRec, all.size() * sizeof(long long), cudaMemcpyDeviceToHost, e->stream);
        st = ce != cudaSuccess ? cuda_fail(ce, "layout record download") : e->wait_stream();
    }
    if (!e->stuck) cudaFree(d);
    NRN_TRY(st);
    for (int r = 0; r < e->world; ++r) {
        const long long* o = all.data() + static_cast<size_t>(r) * kRec;
        for (int k = 0; k < kRec; ++k) {
            if (o[k] == rec[k]) continue;
            comm_destroy(&e->comm, e->comm_timeout_s);
            e->comm_failed = true;
            return fail(NRN_ERR_COMM, "partitioned network: rank " + std::to_string(r) + " and rank " +
                                          std::to_string(e->rank) + " disagree on the spike exchange (layout field " +
                                          std::to_string(k) +
                                          "); every rank must build the same populations, projections, dt, "
                                          "slow ratio and max_rate_hz");
        }
    }
    return NRN_OK;
}

nrn_status_t nrn_engine_add_probe(nrn_engine* e, int32_t pop, int32_t var, float* ring, int32_t depth,
                                  int32_t* id) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(pop >= 0 && pop < static_cast<int32_t>(e->pops.size()), "bad population index");
    NRN_CHECK_ARG(var >= NRN_VAR_V && var <= NRN_VAR_ISYN, "unknown probe variable");
    NRN_CHECK_ARG(ring != nullptr && depth >= 1, "probe: null ring or depth < 1");
    const EnginePop& p = e->pops[pop];
    NRN_CHECK_ARG((var != NRN_VAR_AUX || p.d.aux) && (var != NRN_VAR_REFRACTORY || p.d.refractory),
                  "probe: the population's model has no such variable");
    EngineProbe pr;
    pr.pop = pop;
    pr.var = var;
    pr.ring = ring;
    pr.depth = depth;
    e->probes.push_back(pr);
    e->drop_graphs();
    if (id) *id = static_cast<int32_t>(e->probes.size() - 1);
    return NRN_OK;
}

nrn_status_t nrn_engine_clear_probes(nrn_engine* e) {
    ENGINE_GUARD(e);
    if (!e->probes.empty()) {
        NRN_TRY(e->wait_stream());
        e->probes.clear();
        e->drop_graphs();
    }
    return NRN_OK;
}

nrn_status_t nrn_engine_set_deterministic(nrn_engine* e, int32_t on) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(!e->finalized, "nrn_engine_set_deterministic: call before nrn_engine_finalize");
    NRN_CHECK_ARG(e->world == 1 || !on, "nrn_engine_set_deterministic: deterministic delivery runs on one GPU");
    e->det = on != 0;
    e->drop_graphs();
    return NRN_OK;
}

nrn_status_t nrn_engine_set_comm_timeout(nrn_engine* e, double seconds) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(seconds > 0.0 && std::isfinite(seconds), "nrn_engine_set_comm_timeout: seconds must be positive");
    e->comm_timeout_s = seconds;
    return NRN_OK;
}

nrn_status_t nrn_engine_finalize(nrn_engine* e, int32_t init_update) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(!e->finalized, "engine already finalized");
    int maxd = 1, mind = 255;
    for (auto& q : e->projs) {
        maxd = std::max(maxd, q.csr.dmin + q.csr.nd - 1);
        mind = std::min(mind, q.csr.dmin);
    }
    if (e->projs.empty()) mind = 1;
    for (auto& q : e->projs)
        if (q.plastic) NRN_TRY(build_transpose(q.csr, e->stream));
    if (e->det) {
        NRN_CHECK_ARG(e->world == 1, "deterministic delivery runs on one GPU");
        for (auto& q : e->projs) NRN_TRY(build_det_index(q.csr, e->stream));
        int r = 1;
        while (r < maxd + 1) r <<= 1;
        e->det_ring = r;
        for (auto& p : e->pops) NRN_TRY(dalloc0(&p.flags, static_cast<size_t>(r) * p.n_global, e->stream));
    }
    e->assign_plasticity();
    bool any_walk = false;
    for (auto& q : e->projs) {
        if (q.plastic && !q.walk && e->world > 1)
            return fail(NRN_ERR_UNSUPPORTED,
                        "partitioned network: plasticity needs STDP at every step (slow_ratio 1), at most 256 delays "
                        "and one plastic projection per source population");
        any_walk = any_walk || q.walk;
    }
    // Windows: spikes cross GPUs once per window, and STDP traces are kept at
    // window ends.  A window is at most the smallest delay, so every spike
    // arrives in a later window than the one it was emitted in.
    e->windows = e->world > 1 || any_walk;
    e->win = std::max(1, std::min(mind, 32));
    e->depth = maxd + 1 + (e->world > 1 ? e->win : 0);
    for (auto& p : e->pops) {
        // ring capacity per step: every neuron (one rank), or what all ranks can send
        if (e->world > 1) {
            // Every rank's send block has the same layout (the all-gather moves
            // equal blocks and the unpack reads the other ranks' blocks with
            // this rank's offsets), so it is sized from the largest slice of
            // the population, not from this rank's own slice.
            const double n_max = static_cast<double>((static_cast<int64_t>(p.n_global) + e->world - 1) / e->world);
            const double per_window = std::ceil(n_max * e->win * e->max_rate_hz * e->dt);
            p.send_cap = static_cast<int32_t>(std::min<double>(n_max * e->win, std::max(4096.0, per_window)));
            p.hist_cap = static_cast<int32_t>(std::min<int64_t>(p.n_global,
                                                                static_cast<int64_t>(p.send_cap) * e->world));
        } else {
            p.hist_cap = p.d.n;
        }
        NRN_TRY(dalloc0(&p.hist_ids, static_cast<size_t>(e->depth) * p.hist_cap, e->stream));
        NRN_TRY(dalloc0(&p.hist_count, static_cast<size_t>(e->depth), e->stream));
    }
    if (e->world > 1) {
        e->rank_block = 0;
        for (auto& p : e->pops) {
            p.send_off = e->rank_block;
            e->rank_block += e->win + 1 + p.send_cap;   // [win counts | total | ids]
            e->rank_block = (e->rank_block + 3) / 4 * 4;   // 16-byte aligned blocks
        }
        NRN_TRY(dalloc0(&e->send, static_cast<size_t>(e->rank_block), e->stream));
        NRN_TRY(dalloc0(&e->recv, static_cast<size_t>(e->rank_block) * e->world, e->stream));
        NRN_TRY(check_layout(e));
    }
    int64_t rec_n = 0;
    for (auto& p : e->pops)
        if (p.d.record) rec_n += p.d.n;
    if (rec_n > 0) {
        e->raster_cap = std::max<int64_t>(int64_t(1) << 22, std::min<int64_t>(rec_n * 64, int64_t(1) << 26));
        NRN_TRY(dalloc0(&e->raster_step, e->raster_cap, e->stream));
        NRN_TRY(dalloc0(&e->raster_gid, e->raster_cap, e->stream));
    }
    for (auto& q : e->projs) {
        if (!q.plastic || q.walk) continue;
        NRN_TRY(dalloc0(&q.x_pre, e->pops[q.src_pop].d.n, e->stream));
        NRN_TRY(dalloc0(&q.x_post, e->pops[q.tgt_pop].d.n, e->stream));
    }
    // Walk state.  A segment's T lags the current step by at most about
    // kSweepPeriod + kStale + the window and the delays (the sweep), and a
    // source spike being applied is at most the longest delay old: the
    // snapshot rings are sized for that.
    auto need_history = [&](EnginePop& p) -> nrn_status_t {
        if (p.mask) return NRN_OK;
        NRN_TRY(dalloc0(&p.mask, static_cast<size_t>(p.n_global), e->stream));
        NRN_TRY(dalloc0(&p.recent, static_cast<size_t>(p.n_global) * 4, e->stream));
        NRN_CUDA_TRY(cudaMemsetAsync(p.recent, 0xFF, static_cast<size_t>(p.n_global) * 16, e->stream));   // -1: none
        NRN_TRY(dalloc0(&p.ring, static_cast<size_t>(p.d.n) * kRing, e->stream));
        NRN_TRY(dalloc0(&p.cnt, static_cast<size_t>(p.d.n), e->stream));
        return NRN_OK;
    };
    // target traces: a source spike being applied is at most the longest
    // delay (+1) older than the walk
    auto pow2 = [](int x) {
        int p = 1;
        while (p < x) p <<= 1;
        return p;
    };
    e->ring_depth = pow2(maxd + 2);
    for (auto& q : e->projs) {
        if (!q.walk) continue;
        const size_t nseg = static_cast<size_t>(q.csr.n_src) * q.csr.nd;
        NRN_TRY(dalloc0(&q.work_ctr, 3, e->stream));
        NRN_TRY(dalloc0(&q.seg_last, nseg, e->stream));
        NRN_TRY(dalloc0(&q.seg_x, nseg, e->stream));
        const int dmax = q.csr.dmin + q.csr.nd - 1;
        q.pre_depth = pow2((kSweepPeriod + kStale + e->win + dmax) / e->win + 4);
        NRN_TRY(dalloc0(&q.pre_snap, static_cast<size_t>(q.pre_depth) * q.csr.n_src, e->stream));
        NRN_TRY(dalloc0(&q.post_ring, static_cast<size_t>(e->ring_depth) * q.csr.n_tgt, e->stream));
        NRN_TRY(need_history(e->pops[q.src_pop]));
        NRN_TRY(need_history(e->pops[q.tgt_pop]));
    }
    // The drive is drawn ahead on the side stream (drawing it inside the
    // neuron update, on the critical path, measured 8 us a step slower).
    for (auto& p : e->pops)
        if (p.d.drive.kind != NRN_DRIVE_NONE) NRN_TRY(dalloc0(&p.drive_buf, static_cast<size_t>(p.d.n), e->stream));
    if (e->spike_stats)
        for (auto& p : e->pops) NRN_TRY(dalloc0(&p.stats, static_cast<size_t>(p.d.n), e->stream));
    if (init_update) {
        for (size_t i = 0; i < e->pops.size(); ++i) {
            nrn_pop_step_t a = e->pop_args(static_cast<int>(i), 0.0, 0, false);
            NRN_TRY(nrn_cuda_pop_step(&a, reinterpret_cast<nrn_stream_t>(e->stream)));
        }
    }
    NRN_TRY(e->wait_stream());
    e->finalized = true;
    return NRN_OK;
}

nrn_status_t nrn_engine_prepare(nrn_engine* e, int64_t first_step, int64_t steps, int32_t chunk) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(e->finalized, "nrn_engine_prepare: finalize first");
    NRN_CHECK_ARG(steps >= 0 && first_step >= 0, "nrn_engine_prepare: negative step");
    if (!e->use_graphs || steps == 0) return NRN_OK;
    int64_t s = first_step, left = steps;
    const int w = e->windows ? e->win : 1;
    const int ch = e->run_chunk(chunk);
    while (left > 0) {
        const int phase = static_cast<int>(s % w);
        const int c = e->run_piece(phase, left, ch);
        cudaGraphExec_t g = nullptr;
        NRN_TRY(e->graph_for(c, &g, phase));
        s += c;
        left -= c;
    }
    return NRN_OK;
}

nrn_status_t nrn_engine_run(nrn_engine* e, int64_t steps, int32_t chunk) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(e->finalized, "nrn_engine_run: finalize first");
    NRN_CHECK_ARG(steps >= 0, "negative step count");
    if (e->comm_failed) return fail(NRN_ERR_STATE, "nrn_engine_run: the communicator was aborted after an error");
    if (steps == 0) return NRN_OK;
    NRN_TRY(e->prepare_plastic());
    int64_t s = e->step, left = steps;
    if (!e->use_graphs) {
        for (; left > 0; ++s, --left) NRN_TRY(e->eager_step(s));
    } else {
        // Every step runs inside a graph.  With windows, graphs are keyed by
        // the window phase of their first step: a run that starts inside a
        // window first completes it, then runs whole windows (chunks a
        // multiple of the window), then the rest; the graphs of each shape
        // are captured once and replayed.
        //
        // The steps up to the first window boundary run as one-step graphs,
        // keyed by phase, and a tail shorter than a window as one graph, so a
        // caller whose runs start and stop anywhere meets at most 2w + 2
        // shapes; without windows a tail shorter than a chunk runs as
        // power-of-two graphs.
        const int w = e->windows ? e->win : 1;
        chunk = e->run_chunk(chunk);
        while (left > 0) {
            const int phase = static_cast<int>(s % w);
            const int c = e->run_piece(phase, left, chunk);
            cudaGraphExec_t g = nullptr;
            NRN_TRY(e->graph_for(c, &g, phase));
            NRN_CUDA_TRY(cudaGraphLaunch(g, e->stream));
            s += c;
            left -= c;
        }
    }
    e->step += steps;
    e->step_high = std::max(e->step_high, e->step);
    return NRN_OK;
}

nrn_status_t nrn_engine_profile(nrn_engine* e, int64_t steps, double* ms) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(e->finalized, "nrn_engine_profile: finalize first");
    if (e->comm_failed) return fail(NRN_ERR_STATE, "nrn_engine_profile: the communicator was aborted after an error");
    NRN_CHECK_ARG(steps >= 0 && ms != nullptr, "bad arguments");
    ms[0] = ms[1] = ms[2] = 0.0;
    if (steps == 0) return NRN_OK;
    NRN_TRY(e->prepare_plastic());
    cudaEvent_t ev[4];
    for (auto& x : ev) NRN_CUDA_TRY(cudaEventCreate(&x));
    nrn_status_t st = NRN_OK;
    for (int64_t k = 0; k < steps && st == NRN_OK; ++k) {
        st = e->enqueue_step(0, e->window_end(e->step + k), ev);
        if (st != NRN_OK) break;
        advance_kernel<<<1, 1, 0, e->stream>>>(e->d_step, 1);
        cudaError_t ce = cudaEventSynchronize(ev[3]);
        if (ce != cudaSuccess) { st = cuda_fail(ce, "cudaEventSynchronize"); break; }
        for (int p = 0; p < 3; ++p) {
            float t = 0.0f;
            cudaEventElapsedTime(&t, ev[p], ev[p + 1]);
            ms[p] += t;
        }
    }
    for (auto& x : ev) cudaEventDestroy(x);
    if (st == NRN_OK) {
        NRN_TRY(e->wait_stream());
        e->step += steps;
        e->step_high = std::max(e->step_high, e->step);
    }
    return st;
}

nrn_status_t nrn_engine_profile_kernels(nrn_engine* e, int64_t steps, double* ms, int64_t* counts) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(e->finalized, "nrn_engine_profile_kernels: finalize first");
    NRN_CHECK_ARG(steps >= 0 && ms != nullptr && counts != nullptr, "bad arguments");
    if (e->comm_failed) return fail(NRN_ERR_STATE, "nrn_engine_profile_kernels: the communicator was aborted");
    for (int k = 0; k < 6; ++k) ms[k] = 0.0;
    for (int k = 0; k < 4; ++k) counts[k] = 0;
    if (steps == 0) return NRN_OK;
    NRN_TRY(e->prepare_plastic());
    unsigned long long c0[2] = {0, 0}, c1[2] = {0, 0};
    NRN_CUDA_TRY(cudaMemcpyAsync(c0, e->d_events, sizeof(c0), cudaMemcpyDeviceToHost, e->stream));
    NRN_TRY(e->wait_stream());
    cudaEvent_t ev[7];
    for (auto& x : ev) NRN_CUDA_TRY(cudaEventCreate(&x));
    nrn_status_t st = NRN_OK;
    int64_t wins = 0;
    for (int64_t k = 0; k < steps && st == NRN_OK; ++k) {
        const bool we = e->window_end(e->step + k);
        wins += we ? 1 : 0;
        st = e->enqueue_step(0, we, nullptr, ev);
        if (st != NRN_OK) break;
        advance_kernel<<<1, 1, 0, e->stream>>>(e->d_step, 1);
        cudaError_t ce = cudaEventSynchronize(ev[6]);
        if (ce != cudaSuccess) { st = cuda_fail(ce, "cudaEventSynchronize"); break; }
        for (int p = 0; p < 6; ++p) {
            float t = 0.0f;
            cudaEventElapsedTime(&t, ev[p], ev[p + 1]);
            ms[p] += t;
        }
    }
    for (auto& x : ev) cudaEventDestroy(x);
    if (st == NRN_OK) {
        NRN_CUDA_TRY(cudaMemcpyAsync(c1, e->d_events, sizeof(c1), cudaMemcpyDeviceToHost, e->stream));
        NRN_TRY(e->wait_stream());
        e->step += steps;
        e->step_high = std::max(e->step_high, e->step);
        counts[0] = static_cast<int64_t>(c1[0] - c0[0]);
        counts[1] = static_cast<int64_t>(c1[1] - c0[1]);
        counts[2] = wins;
        counts[3] = steps;
    }
    return st;
}

nrn_status_t nrn_engine_set_step(nrn_engine* e, int64_t step) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(step >= 0, "step must be >= 0");
    const long long s = step;
    NRN_CUDA_TRY(cudaMemcpyAsync(e->d_step, &s, sizeof(s), cudaMemcpyHostToDevice, e->stream));
    NRN_TRY(e->wait_stream());
    e->step = step;
    e->step_high = std::max(e->step_high, e->step);
    return NRN_OK;
}

nrn_status_t nrn_engine_sync(nrn_engine* e) {
    ENGINE_GUARD(e);
    NRN_TRY(e->wait_stream());
    return e->check_err();
}

nrn_status_t nrn_engine_raster(nrn_engine* e, int32_t* step, int32_t* gid, int64_t cap, int64_t* n) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(n != nullptr, "null count");
    unsigned long long cnt = 0;
    NRN_CUDA_TRY(cudaMemcpyAsync(&cnt, e->d_raster_count, sizeof(cnt), cudaMemcpyDeviceToHost, e->stream));
    NRN_TRY(e->wait_stream());
    *n = static_cast<int64_t>(cnt);
    if (cnt == 0) return NRN_OK;
    if (static_cast<int64_t>(cnt) > e->raster_cap)
        return fail(NRN_ERR_CAPACITY, "spike raster overflowed: read it more often (" + std::to_string(cnt) +
                                          " spikes, capacity " + std::to_string(e->raster_cap) + ")");
    if (static_cast<int64_t>(cnt) > cap) return fail(NRN_ERR_CAPACITY, "output buffer too small for the raster");
    // order of the reference's recorder: by step, ascending ids within a step
    int64_t total = 0;
    for (const auto& p : e->pops) total += p.n_global;
    auto bits_for = [](int64_t max_value) {   // bits that hold 0 .. max_value
        int b = 1;
        while (b < 62 && (int64_t(1) << b) <= max_value) ++b;
        return b;
    };
    NRN_TRY(sort_raster(e->raster_step, e->raster_gid, static_cast<int64_t>(cnt), bits_for(total - 1),
                        bits_for(std::max<int64_t>(e->step_high, 1)), e->sort_scratch, e->stream));
    NRN_CUDA_TRY(cudaMemcpyAsync(step, e->raster_step, cnt * 4, cudaMemcpyDeviceToHost, e->stream));
    NRN_CUDA_TRY(cudaMemcpyAsync(gid, e->raster_gid, cnt * 4, cudaMemcpyDeviceToHost, e->stream));
    NRN_CUDA_TRY(cudaMemsetAsync(e->d_raster_count, 0, sizeof(unsigned long long), e->stream));
    NRN_TRY(e->wait_stream());
    e->spikes_flushed += static_cast<int64_t>(cnt);
    return NRN_OK;
}

nrn_status_t nrn_engine_nnz(nrn_engine* e, int32_t proj, int64_t* nnz) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(proj >= 0 && proj < static_cast<int32_t>(e->projs.size()) && nnz, "bad projection index");
    *nnz = e->projs[proj].csr.nnz;
    return NRN_OK;
}

nrn_status_t nrn_engine_weights(nrn_engine* e, int32_t proj, float* out, int64_t n) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(proj >= 0 && proj < static_cast<int32_t>(e->projs.size()), "bad projection index");
    const auto& c = e->projs[proj].csr;
    NRN_CHECK_ARG(n == c.nnz && out != nullptr, "weights: output size must equal the synapse count");
    NRN_TRY(e->flush_walks());
    NRN_TRY(e->check_err());
    std::vector<float> w(static_cast<size_t>(c.nnz));
    NRN_TRY(e->wait_stream());
    if (c.nnz) NRN_CUDA_TRY(cudaMemcpy(w.data(), c.w, c.nnz * 4, cudaMemcpyDeviceToHost));
    if (c.orig) {
        std::vector<int64_t> o(static_cast<size_t>(c.nnz));
        if (c.nnz) NRN_CUDA_TRY(cudaMemcpy(o.data(), c.orig, c.nnz * 8, cudaMemcpyDeviceToHost));
        for (int64_t k = 0; k < c.nnz; ++k) out[o[k]] = w[k];
    } else {
        std::memcpy(out, w.data(), c.nnz * 4);
    }
    return NRN_OK;
}

nrn_status_t nrn_engine_weights_device(nrn_engine* e, int32_t proj, float* out, int64_t n) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(proj >= 0 && proj < static_cast<int32_t>(e->projs.size()), "bad projection index");
    const auto& c = e->projs[proj].csr;
    NRN_CHECK_ARG(n == c.nnz && (n == 0 || out != nullptr), "weights: output size must equal the synapse count");
    if (n == 0) return NRN_OK;
    NRN_TRY(e->flush_walks());
    NRN_TRY(e->check_err());
    if (c.orig) {
        // out[orig[k]] = w[k]
        return nrn_cuda_scatter(c.w, c.orig, n, out, reinterpret_cast<nrn_stream_t>(e->stream));
    }
    NRN_CUDA_TRY(cudaMemcpyAsync(out, c.w, n * sizeof(float), cudaMemcpyDeviceToDevice, e->stream));
    return NRN_OK;
}

nrn_status_t nrn_engine_set_state(nrn_engine* e, int32_t pop, float* v, float* aux, float* refractory, float* spike,
                                  float* i_syn) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(pop >= 0 && pop < static_cast<int32_t>(e->pops.size()), "bad population index");
    auto& p = e->pops[pop];
    NRN_CHECK_ARG(v && spike, "population needs v and spike arrays");
    NRN_CHECK_ARG(p.d.model == NRN_MODEL_LIF || aux, "population needs aux (w/u)");
    NRN_CHECK_ARG(p.d.model == NRN_MODEL_IZH || refractory, "population needs refractory");
    bool changed = v != p.d.v || aux != p.d.aux || refractory != p.d.refractory || spike != p.d.spike;
    p.d.v = v;
    p.d.aux = aux;
    p.d.refractory = refractory;
    p.d.spike = spike;
    if (i_syn != nullptr && i_syn != p.d.i_syn) {
        if (p.owns_isyn) cudaFree(p.d.i_syn);
        p.owns_isyn = false;
        p.d.i_syn = i_syn;
        changed = true;
    }
    if (changed) e->drop_graphs();
    return NRN_OK;
}

nrn_status_t nrn_engine_counters(nrn_engine* e, int64_t* spikes, int64_t* events) {
    ENGINE_GUARD(e);
    unsigned long long ev2[2] = {0, 0}, rc = 0;
    NRN_CUDA_TRY(cudaMemcpyAsync(ev2, e->d_events, sizeof(ev2), cudaMemcpyDeviceToHost, e->stream));
    NRN_CUDA_TRY(cudaMemcpyAsync(&rc, e->d_raster_count, sizeof(rc), cudaMemcpyDeviceToHost, e->stream));
    NRN_TRY(e->wait_stream());
    if (events) *events = static_cast<int64_t>(ev2[0] + ev2[1]);
    if (spikes) *spikes = e->spikes_flushed + static_cast<int64_t>(rc);
    return NRN_OK;
}

namespace {

size_t ckpt_bytes(const std::vector<nrn_engine::StateBuf>& b, size_t n_proj, int64_t raster_n) {
    size_t s = sizeof(CkptHeader) + 8 * b.size() + (n_proj + 7) / 8 * 8;
    for (const auto& x : b) s += x.bytes;
    return s + 8 * static_cast<size_t>(raster_n);
}

// The engine can be checkpointed now: finalized, no error pending, and for
// a partitioned engine at a window boundary.  *raster_n: spikes recorded
// and not yet read.
nrn_status_t ckpt_ready(nrn_engine* e, int64_t* raster_n) {
    NRN_CHECK_ARG(e->finalized, "checkpoint: finalize the engine first");
    if (e->world > 1 && e->step % e->win != 0)
        return fail(NRN_ERR_STATE, "checkpoint: a partitioned engine is checkpointed at window boundaries (step " +
                                       std::to_string(e->step) + ", window " + std::to_string(e->win) + ")");
    NRN_TRY(e->check_err());
    unsigned long long rc = 0;
    NRN_CUDA_TRY(cudaMemcpyAsync(&rc, e->d_raster_count, sizeof(rc), cudaMemcpyDeviceToHost, e->stream));
    NRN_TRY(e->wait_stream());
    if (static_cast<int64_t>(rc) > e->raster_cap)
        return fail(NRN_ERR_CAPACITY, "checkpoint: the spike raster overflowed; read it first");
    *raster_n = static_cast<int64_t>(rc);
    return NRN_OK;
}

}  // namespace

nrn_status_t nrn_engine_enable_spike_stats(nrn_engine* e) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(!e->finalized, "enable_spike_stats: call before nrn_engine_finalize");
    e->spike_stats = true;
    return NRN_OK;
}

nrn_status_t nrn_engine_spike_stats(nrn_engine* e, int32_t pop, nrn_spike_stat_t* out, int64_t n) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(pop >= 0 && pop < static_cast<int32_t>(e->pops.size()), "bad population index");
    const auto& p = e->pops[pop];
    if (p.stats == nullptr) return fail(NRN_ERR_STATE, "spike statistics were not enabled before finalize");
    NRN_CHECK_ARG(n == p.d.n && out != nullptr, "spike_stats: output size must equal the population's local size");
    NRN_CUDA_TRY(cudaMemcpyAsync(out, p.stats, static_cast<size_t>(n) * sizeof(nrn_spike_stat_t),
                                 cudaMemcpyDeviceToHost, e->stream));
    NRN_TRY(e->wait_stream());
    return NRN_OK;
}

nrn_status_t nrn_engine_spike_stats_reset(nrn_engine* e) {
    ENGINE_GUARD(e);
    if (!e->spike_stats || !e->finalized) return fail(NRN_ERR_STATE, "spike statistics are not enabled");
    for (const auto& p : e->pops)
        NRN_CUDA_TRY(cudaMemsetAsync(p.stats, 0, static_cast<size_t>(p.d.n) * sizeof(nrn_spike_stat_t), e->stream));
    NRN_TRY(e->wait_stream());
    return NRN_OK;
}

nrn_status_t nrn_engine_checkpoint_size(nrn_engine* e, int64_t* bytes) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(bytes != nullptr, "checkpoint_size: null output");
    int64_t rn = 0;
    NRN_TRY(ckpt_ready(e, &rn));
    *bytes = static_cast<int64_t>(ckpt_bytes(e->state_buffers(), e->projs.size(), rn));
    return NRN_OK;
}

nrn_status_t nrn_engine_checkpoint_save(nrn_engine* e, void* buf, int64_t bytes) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(buf != nullptr, "checkpoint_save: null buffer");
    int64_t rn = 0;
    NRN_TRY(ckpt_ready(e, &rn));
    const auto b = e->state_buffers();
    const size_t n_proj = e->projs.size();
    NRN_CHECK_ARG(bytes == static_cast<int64_t>(ckpt_bytes(b, n_proj, rn)),
                  "checkpoint_save: buffer size differs from nrn_engine_checkpoint_size");
    char* out = static_cast<char*>(buf);
    CkptHeader h{};
    std::memcpy(h.magic, kCkptMagic, sizeof(h.magic));
    h.step = e->step;
    h.spikes_flushed = e->spikes_flushed;
    h.raster_n = rn;
    h.world = e->world;
    h.rank = e->rank;
    h.n_buf = static_cast<int32_t>(b.size());
    h.n_proj = static_cast<int32_t>(n_proj);
    std::memcpy(out, &h, sizeof(h));
    out += sizeof(h);
    for (const auto& x : b) {
        const uint64_t sz = x.bytes;
        std::memcpy(out, &sz, 8);
        out += 8;
    }
    std::memset(out, 0, (n_proj + 7) / 8 * 8);
    for (size_t q = 0; q < n_proj; ++q) out[q] = e->projs[q].clamped ? 1 : 0;
    out += (n_proj + 7) / 8 * 8;
    for (const auto& x : b) {
        NRN_CUDA_TRY(cudaMemcpyAsync(out, x.p, x.bytes, cudaMemcpyDeviceToHost, e->stream));
        out += x.bytes;
    }
    if (rn > 0) {
        NRN_CUDA_TRY(cudaMemcpyAsync(out, e->raster_step, rn * 4, cudaMemcpyDeviceToHost, e->stream));
        NRN_CUDA_TRY(cudaMemcpyAsync(out + rn * 4, e->raster_gid, rn * 4, cudaMemcpyDeviceToHost, e->stream));
    }
    NRN_TRY(e->wait_stream());
    return NRN_OK;
}

nrn_status_t nrn_engine_checkpoint_load(nrn_engine* e, const void* buf, int64_t bytes) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(e->finalized, "checkpoint_load: finalize the engine first");
    NRN_CHECK_ARG(buf != nullptr && bytes >= static_cast<int64_t>(sizeof(CkptHeader)), "checkpoint_load: not a checkpoint");
    const char* in = static_cast<const char*>(buf);
    CkptHeader h;
    std::memcpy(&h, in, sizeof(h));
    NRN_CHECK_ARG(std::memcmp(h.magic, kCkptMagic, sizeof(h.magic)) == 0, "checkpoint_load: not a checkpoint");
    NRN_CHECK_ARG(h.world == e->world && h.rank == e->rank,
                  "checkpoint_load: taken by another rank or with another number of GPUs");
    const auto b = e->state_buffers();
    const size_t n_proj = e->projs.size();
    NRN_CHECK_ARG(h.n_buf == static_cast<int32_t>(b.size()) && h.n_proj == static_cast<int32_t>(n_proj) &&
                      h.raster_n >= 0 && h.raster_n <= e->raster_cap && h.step >= 0,
                  "checkpoint_load: the checkpoint is of another network");
    NRN_CHECK_ARG(bytes == static_cast<int64_t>(ckpt_bytes(b, n_proj, h.raster_n)),
                  "checkpoint_load: the checkpoint is of another network (size)");
    in += sizeof(h);
    for (const auto& x : b) {
        uint64_t sz = 0;
        std::memcpy(&sz, in, 8);
        in += 8;
        NRN_CHECK_ARG(sz == x.bytes, "checkpoint_load: the checkpoint is of another network (buffer sizes)");
    }
    NRN_TRY(e->wait_stream());
    for (size_t q = 0; q < n_proj; ++q) e->projs[q].clamped = in[q] != 0;
    in += (n_proj + 7) / 8 * 8;
    for (const auto& x : b) {
        NRN_CUDA_TRY(cudaMemcpyAsync(x.p, in, x.bytes, cudaMemcpyHostToDevice, e->stream));
        in += x.bytes;
    }
    const unsigned long long rc = static_cast<unsigned long long>(h.raster_n);
    NRN_CUDA_TRY(cudaMemcpyAsync(e->d_raster_count, &rc, sizeof(rc), cudaMemcpyHostToDevice, e->stream));
    if (h.raster_n > 0) {
        NRN_CUDA_TRY(cudaMemcpyAsync(e->raster_step, in, h.raster_n * 4, cudaMemcpyHostToDevice, e->stream));
        NRN_CUDA_TRY(cudaMemcpyAsync(e->raster_gid, in + h.raster_n * 4, h.raster_n * 4, cudaMemcpyHostToDevice,
                                     e->stream));
    }
    const long long st = h.step;
    NRN_CUDA_TRY(cudaMemcpyAsync(e->d_step, &st, sizeof(st), cudaMemcpyHostToDevice, e->stream));
    NRN_CUDA_TRY(cudaMemsetAsync(e->d_err, 0, sizeof(int), e->stream));
    NRN_TRY(e->wait_stream());
    e->step = h.step;
    e->step_high = std::max(e->step_high, e->step);
    e->spikes_flushed = h.spikes_flushed;
    return NRN_OK;
}

}  // extern "C"
