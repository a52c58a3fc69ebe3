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
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
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
    bool cond = false;
    bool owns_isyn = false;
    float* g_exc = nullptr;
    float* g_inh = nullptr;
    float* gin_exc = nullptr;
    float* gin_inh = nullptr;
    int32_t* hist_ids = nullptr;
    int32_t* hist_count = nullptr;
    // spike-time history for deferred plasticity (target of a deferred projection)
    int32_t* post_recent = nullptr;   // [n][4]
    int32_t* post_ring = nullptr;     // [n][kPostRing]
    int32_t* post_cnt = nullptr;      // [n]
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
    bool deferred = false;       // potentiation deferred to row passes (plastic.cu)
    int32_t* seg_last = nullptr;
    float* seg_x = nullptr;
    float* x_snap = nullptr;
};

constexpr int kPostRing = 64;       // target spike steps kept per neuron
constexpr int kSnapPeriod = 16;     // steps between x_pre snapshots
constexpr int kSnapDepth = 64;      // snapshots kept
constexpr int kSweepPeriod = 960;   // every row is walked at least this often (< (depth-1)*period)

struct nrn_engine {
    int device = 0;
    double dt = 1e-4;
    int32_t slow_ratio = 1;
    cudaStream_t stream = nullptr;
    std::vector<EnginePop> pops;
    std::vector<EngineProj> projs;
    bool finalized = false;
    int32_t depth = 2;
    int64_t step = 0;                     // host mirror of the device step
    long long* d_step = nullptr;          // device step base
    unsigned long long* d_events = nullptr;
    unsigned long long* d_raster_count = nullptr;
    int32_t* raster_step = nullptr;
    int32_t* raster_gid = nullptr;
    int64_t raster_cap = 0;
    int64_t spikes_flushed = 0;
    std::map<int, cudaGraphExec_t> graphs;
    int* d_err = nullptr;                 // deferred-plasticity history overflow

    ~nrn_engine() {
        if (device >= 0) cudaSetDevice(device);
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        for (auto& p : pops) {
            if (p.owns_isyn) cudaFree(p.d.i_syn);
            cudaFree(p.g_exc); cudaFree(p.g_inh); cudaFree(p.gin_exc); cudaFree(p.gin_inh);
            cudaFree(p.hist_ids); cudaFree(p.hist_count);
            cudaFree(p.post_recent); cudaFree(p.post_ring); cudaFree(p.post_cnt);
        }
        for (auto& q : projs) {
            free_csr(q.csr);
            cudaFree(q.x_pre);
            cudaFree(q.x_post);
            cudaFree(q.seg_last); cudaFree(q.seg_x); cudaFree(q.x_snap);
        }
        cudaFree(d_step); cudaFree(d_events); cudaFree(d_raster_count); cudaFree(d_err);
        cudaFree(raster_step); cudaFree(raster_gid);
        if (stream) cudaStreamDestroy(stream);
    }

    float* acc_of(const EngineProj& q) const {
        const EnginePop& t = pops[q.tgt_pop];
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
        h.cap = pops[i].d.n > 0 ? pops[i].d.n : 1;
        h.depth = depth;
        return h;
    }

    nrn_pop_step_t pop_args(int i, double dt_step, int64_t step_off, bool in_run) const {
        const EnginePop& p = pops[i];
        nrn_pop_step_t a{};
        a.model = p.d.model;
        a.n = p.d.n;
        a.gid_offset = p.d.gid_offset;
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
            a.drive = p.d.drive;
            a.step = step_off;
            a.step_base = reinterpret_cast<const int64_t*>(d_step);
            a.spike_ids = p.hist_ids;
            a.spike_count = p.hist_count;
            a.hist_depth = depth;
            a.hist_cap = p.d.n > 0 ? p.d.n : 1;
            if (p.d.record) {
                a.raster_step = raster_step;
                a.raster_gid = raster_gid;
                a.raster_count = d_raster_count;
                a.raster_cap = raster_cap;
            }
            // plasticity traces of the projections this population feeds or receives
            a.trace_slow_ratio = slow_ratio;
            a.snap_trace = -1;
            for (const auto& q : projs) {
                if (!q.plastic || !q.traces_fused) continue;
                if (q.src_pop == i) {
                    if (q.deferred) {
                        a.snap_trace = a.n_traces;
                        a.snap_buf = q.x_snap;
                        a.snap_period = kSnapPeriod;
                        a.snap_depth = kSnapDepth;
                    }
                    a.trace[a.n_traces] = q.x_pre;
                    a.trace_decay[a.n_traces++] = static_cast<float>(std::exp(-dt / q.stdp[0]));
                }
                if (q.tgt_pop == i) {
                    a.trace[a.n_traces] = q.x_post;
                    a.trace_decay[a.n_traces++] = static_cast<float>(std::exp(-dt / q.stdp[1]));
                }
            }
            if (p.post_recent) {
                a.post_recent = p.post_recent;
                a.post_ring = p.post_ring;
                a.post_cnt = p.post_cnt;
                a.post_ring_k = kPostRing;
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

    PlasticArgs plastic_args(const EngineProj& q) const {
        PlasticArgs a;
        a.n_src = q.csr.n_src;
        a.nd = q.csr.nd;
        a.dmin = q.csr.dmin;
        a.seg_ptr = q.csr.seg_ptr;
        a.tgt = q.csr.tgt;
        a.w = q.csr.w;
        a.mod = q.csr.mod;
        a.acc = acc_of(q);
        a.x_pre = q.x_pre;
        a.x_post = q.x_post;
        a.spike_src = pops[q.src_pop].d.spike;
        a.spike_tgt = pops[q.tgt_pop].d.spike;
        a.hist_src = hist(q.src_pop);
        a.a_plus = static_cast<float>(q.stdp[2]);
        a.a_minus = static_cast<float>(std::fabs(q.stdp[3]));
        a.lr = static_cast<float>(q.stdp[6]);
        a.w_min = static_cast<float>(q.stdp[4]);
        a.w_max = static_cast<float>(q.stdp[5]);
        a.decay_pre = static_cast<float>(std::exp(-dt / q.stdp[0]));
        a.seg_last = q.seg_last;
        a.seg_x = q.seg_x;
        a.x_snap = q.x_snap;
        a.snap_period = kSnapPeriod;
        a.snap_depth = kSnapDepth;
        const EnginePop& t = pops[q.tgt_pop];
        a.post_recent = reinterpret_cast<const int4*>(t.post_recent);
        a.post_ring = t.post_ring;
        a.post_cnt = t.post_cnt;
        a.post_ring_k = kPostRing;
        a.sweep_period = kSweepPeriod;
        a.sweep_rows = (q.csr.n_src + kSweepPeriod - 1) / kSweepPeriod;
        a.err = d_err;
        a.events = d_events;
        return a;
    }

    // Walks every row of the deferred projections so that their weights are
    // up to date through the last step run (before weights are read).
    nrn_status_t flush_deferred() {
        if (step <= 0) return NRN_OK;
        for (auto& q : projs)
            if (q.deferred) NRN_TRY(plastic_rows(plastic_args(q), PLASTIC_FLUSH, step - 1, nullptr, stream));
        return NRN_OK;
    }

    nrn_status_t check_err() {
        int h = 0;
        NRN_CUDA_TRY(cudaMemcpyAsync(&h, d_err, sizeof(int), cudaMemcpyDeviceToHost, stream));
        NRN_CUDA_TRY(cudaStreamSynchronize(stream));
        if (h == 1) return fail(NRN_ERR_CAPACITY, "STDP: a target spiked more often than its spike history holds");
        if (h == 2) return fail(NRN_ERR_STATE, "STDP: a row was not refreshed within the trace snapshot window");
        return NRN_OK;
    }

    // Decides, per plastic projection, whether the neuron updates of its
    // source and target advance its traces (both or neither: a projection
    // that does not fit in the NRN_MAX_TRACES slots of both populations
    // keeps the separate trace kernel).
    void assign_trace_slots() {
        std::vector<int> used(pops.size(), 0);
        for (auto& q : projs) {
            q.traces_fused = false;
            if (!q.plastic) continue;
            const int need_src = 1 + (q.src_pop == q.tgt_pop ? 1 : 0);
            if (q.src_pop == q.tgt_pop) {
                if (used[q.src_pop] + need_src <= NRN_MAX_TRACES) {
                    used[q.src_pop] += 2;
                    q.traces_fused = true;
                }
            } else if (used[q.src_pop] < NRN_MAX_TRACES && used[q.tgt_pop] < NRN_MAX_TRACES) {
                used[q.src_pop] += 1;
                used[q.tgt_pop] += 1;
                q.traces_fused = true;
            }
        }
        // Deferred potentiation needs STDP on every step, fused traces and one
        // snapshot slot per source population.
        std::vector<char> snap_used(pops.size(), 0);
        for (auto& q : projs) {
            q.deferred = false;
            if (!q.plastic || !q.traces_fused || slow_ratio != 1 || q.csr.nd > 256) continue;
            if (snap_used[q.src_pop]) continue;
            snap_used[q.src_pop] = 1;
            q.deferred = true;
        }
    }

    // Enqueues one step at offset `off` from *d_step; with `ev` non-null,
    // records events around the three phases (ev[0..3]).
    nrn_status_t enqueue_step(int64_t off, cudaEvent_t* ev = nullptr) {
        std::vector<nrn_proj_t> dp;
        std::vector<int> src_map;
        for (auto& q : projs)
            if (!q.deferred) dp.push_back(dev_proj(q));
        std::vector<nrn_spike_hist_t> hs;
        for (size_t i = 0; i < pops.size(); ++i) hs.push_back(hist(static_cast<int>(i)));
        if (ev) NRN_CUDA_TRY(cudaEventRecord(ev[0], stream));
        NRN_TRY(nrn_cuda_deliver_counted(dp.data(), static_cast<int32_t>(dp.size()), hs.data(),
                                         static_cast<int32_t>(hs.size()), off,
                                         reinterpret_cast<const int64_t*>(d_step), d_events,
                                         reinterpret_cast<nrn_stream_t>(stream)));
        for (auto& q : projs)
            if (q.deferred) NRN_TRY(plastic_rows(plastic_args(q), PLASTIC_DELIVER, off, d_step, stream));
        if (ev) NRN_CUDA_TRY(cudaEventRecord(ev[1], stream));
        for (size_t i = 0; i < pops.size(); ++i) {
            nrn_pop_step_t a = pop_args(static_cast<int>(i), dt, off, true);
            NRN_TRY(nrn_cuda_pop_step(&a, reinterpret_cast<nrn_stream_t>(stream)));
        }
        if (ev) NRN_CUDA_TRY(cudaEventRecord(ev[2], stream));
        for (auto& q : projs) {
            if (!q.plastic) continue;
            if (q.deferred) {
                NRN_TRY(plastic_rows(plastic_args(q), PLASTIC_LTD, off, d_step, stream));
                continue;
            }
            nrn_stdp_t s = stdp_args(q);
            NRN_TRY(nrn_cuda_stdp_step(&s, off, reinterpret_cast<const int64_t*>(d_step),
                                        reinterpret_cast<nrn_stream_t>(stream)));
        }
        if (ev) NRN_CUDA_TRY(cudaEventRecord(ev[3], stream));
        return NRN_OK;
    }

    nrn_status_t graph_for(int chunk, cudaGraphExec_t* out) {
        auto it = graphs.find(chunk);
        if (it != graphs.end()) {
            *out = it->second;
            return NRN_OK;
        }
        cudaGraph_t g = nullptr;
        NRN_CUDA_TRY(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
        nrn_status_t st = NRN_OK;
        for (int k = 0; k < chunk && st == NRN_OK; ++k) st = enqueue_step(k);
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
        graphs[chunk] = ex;
        *out = ex;
        return NRN_OK;
    }

    void drop_graphs() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        graphs.clear();
    }
};

#define ENGINE_GUARD(e)                                                          \
    do {                                                                         \
        if ((e) == nullptr) return fail(NRN_ERR_INVALID, "null engine");         \
        cudaError_t ce_ = cudaSetDevice((e)->device);                            \
        if (ce_ != cudaSuccess) return cuda_fail(ce_, "cudaSetDevice");          \
    } while (0)

namespace nrn {

nrn_status_t engine_raster_view(nrn_engine* e, EngineRasterView* v) {
    NRN_CHECK_ARG(e != nullptr && v != nullptr, "null engine");
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
    NRN_CUDA_TRY(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    NRN_TRY(dalloc0(&e->d_step, 1, e->stream));
    NRN_TRY(dalloc0(&e->d_events, 1, e->stream));
    NRN_TRY(dalloc0(&e->d_raster_count, 1, e->stream));
    NRN_TRY(dalloc0(&e->d_err, 1, e->stream));
    *out = e.release();
    return NRN_OK;
}

nrn_status_t nrn_engine_destroy(nrn_engine* e) {
    if (e == nullptr) return NRN_OK;
    cudaSetDevice(e->device);
    cudaStreamSynchronize(e->stream);
    delete e;
    return NRN_OK;
}

nrn_status_t nrn_engine_stream(nrn_engine* e, nrn_stream_t* stream) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(stream != nullptr, "null output");
    *stream = reinterpret_cast<nrn_stream_t>(e->stream);
    return NRN_OK;
}

int64_t nrn_engine_step(const nrn_engine* e) { return e ? e->step : -1; }

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
    NRN_TRY(build_csr(q.csr, e->pops[src_pop].d.n, e->pops[tgt_pop].d.n, src, tgt, w, delay, mod, n, keep_orig,
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
    NRN_CHECK_ARG(d->receptor >= NRN_RECV_CURRENT && d->receptor <= NRN_RECV_GINH, "bad receptor");
    NRN_CHECK_ARG(d->receptor == NRN_RECV_CURRENT || e->pops[d->tgt_pop].cond,
                  "conductance receptor on a population without conductance input");
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
    cudaStreamSynchronize(e->stream);
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
    NRN_CHECK_ARG(g->receptor == NRN_RECV_CURRENT || e->pops[g->tgt_pop].cond,
                  "conductance receptor on a population without conductance input");
    const auto& ps = e->pops[g->src_pop].d;
    const auto& pt = e->pops[g->tgt_pop].d;
    GenArgs a{};
    a.out_degree = g->out_degree;
    a.degree = g->degree;
    a.gen_id = static_cast<uint32_t>(g->gen_id);
    a.n_src = ps.n;
    a.src_offset = ps.gid_offset;
    a.col_offset = g->col_n > 0 ? g->col_offset : (g->out_degree ? pt.gid_offset : ps.gid_offset);
    a.col_n = g->col_n > 0 ? g->col_n : (g->out_degree ? pt.n : ps.n);
    a.row_offset = g->out_degree ? ps.gid_offset : pt.gid_offset;
    a.n_rows = g->out_degree ? ps.n : pt.n;
    a.keep_lo = pt.gid_offset;
    a.keep_hi = pt.gid_offset + pt.n;
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
    cudaStreamSynchronize(e->stream);
    cleanup();
    if (st == NRN_OK && nnz) *nnz = e->projs.back().csr.nnz;
    return st;
}

nrn_status_t nrn_engine_set_stdp(nrn_engine* e, int32_t proj, const double* p) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(proj >= 0 && proj < static_cast<int32_t>(e->projs.size()), "bad projection index");
    NRN_CHECK_ARG(p != nullptr, "null STDP parameters");
    NRN_CHECK_ARG(p[0] > 0 && p[1] > 0, "STDP time constants must be positive");
    NRN_CHECK_ARG(p[4] <= p[5], "STDP needs w_min <= w_max");
    NRN_CHECK_ARG(!e->finalized, "nrn_engine_set_stdp: set plasticity before nrn_engine_finalize");
    auto& q = e->projs[proj];
    std::memcpy(q.stdp, p, sizeof(q.stdp));
    q.plastic = true;
    e->drop_graphs();
    return NRN_OK;
}

nrn_status_t nrn_engine_finalize(nrn_engine* e, int32_t init_update) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(!e->finalized, "engine already finalized");
    int maxd = 1;
    for (auto& q : e->projs) maxd = std::max(maxd, q.csr.dmin + q.csr.nd - 1);
    e->depth = maxd + 1;
    for (auto& p : e->pops) {
        NRN_TRY(dalloc0(&p.hist_ids, static_cast<size_t>(e->depth) * p.d.n, e->stream));
        NRN_TRY(dalloc0(&p.hist_count, static_cast<size_t>(e->depth), e->stream));
    }
    int64_t rec_n = 0;
    for (auto& p : e->pops)
        if (p.d.record) rec_n += p.d.n;
    if (rec_n > 0) {
        e->raster_cap = std::max<int64_t>(int64_t(1) << 20, std::min<int64_t>(rec_n * 64, int64_t(1) << 26));
        NRN_TRY(dalloc0(&e->raster_step, e->raster_cap, e->stream));
        NRN_TRY(dalloc0(&e->raster_gid, e->raster_cap, e->stream));
    }
    for (auto& q : e->projs) {
        if (!q.plastic) continue;
        NRN_TRY(build_transpose(q.csr, e->stream));
        NRN_TRY(dalloc0(&q.x_pre, e->pops[q.src_pop].d.n, e->stream));
        NRN_TRY(dalloc0(&q.x_post, e->pops[q.tgt_pop].d.n, e->stream));
    }
    e->assign_trace_slots();
    for (auto& q : e->projs) {
        if (!q.deferred) continue;
        const size_t nseg = static_cast<size_t>(q.csr.n_src) * q.csr.nd;
        NRN_TRY(dalloc0(&q.seg_last, nseg, e->stream));
        NRN_CUDA_TRY(cudaMemsetAsync(q.seg_last, 0xFF, nseg * sizeof(int32_t), e->stream));   // -1: nothing applied
        NRN_TRY(dalloc0(&q.seg_x, nseg, e->stream));
        NRN_TRY(dalloc0(&q.x_snap, static_cast<size_t>(kSnapDepth) * q.csr.n_src, e->stream));
        auto& t = e->pops[q.tgt_pop];
        if (!t.post_recent) {
            NRN_TRY(dalloc0(&t.post_recent, static_cast<size_t>(t.d.n) * 4, e->stream));
            NRN_CUDA_TRY(cudaMemsetAsync(t.post_recent, 0xFF, static_cast<size_t>(t.d.n) * 16, e->stream));
            NRN_TRY(dalloc0(&t.post_ring, static_cast<size_t>(t.d.n) * kPostRing, e->stream));
            NRN_TRY(dalloc0(&t.post_cnt, static_cast<size_t>(t.d.n), e->stream));
        }
    }
    if (init_update) {
        for (size_t i = 0; i < e->pops.size(); ++i) {
            nrn_pop_step_t a = e->pop_args(static_cast<int>(i), 0.0, 0, false);
            NRN_TRY(nrn_cuda_pop_step(&a, reinterpret_cast<nrn_stream_t>(e->stream)));
        }
    }
    NRN_CUDA_TRY(cudaStreamSynchronize(e->stream));
    e->finalized = true;
    return NRN_OK;
}

nrn_status_t nrn_engine_run(nrn_engine* e, int64_t steps, int32_t chunk) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(e->finalized, "nrn_engine_run: finalize first");
    NRN_CHECK_ARG(steps >= 0, "negative step count");
    if (steps == 0) return NRN_OK;
    // The reference clamps every weight of a plastic connection on each
    // update (stdp.cpp:139); one clamp of all weights before the first
    // update, then of each changed weight, is the same.
    for (auto& q : e->projs) {
        if (q.plastic && !q.clamped) {
            NRN_TRY(nrn_cuda_clamp(q.csr.w, q.csr.nnz, static_cast<float>(q.stdp[4]), static_cast<float>(q.stdp[5]),
                                   reinterpret_cast<nrn_stream_t>(e->stream)));
            q.clamped = true;
        }
    }
    if (chunk <= 0) chunk = static_cast<int32_t>(std::min<int64_t>(steps, 50));
    int64_t done = 0;
    while (done < steps) {
        const int c = static_cast<int>(std::min<int64_t>(chunk, steps - done));
        cudaGraphExec_t g = nullptr;
        NRN_TRY(e->graph_for(c, &g));
        NRN_CUDA_TRY(cudaGraphLaunch(g, e->stream));
        done += c;
    }
    e->step += steps;
    return NRN_OK;
}

nrn_status_t nrn_engine_profile(nrn_engine* e, int64_t steps, double* ms) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(e->finalized, "nrn_engine_profile: finalize first");
    NRN_CHECK_ARG(steps >= 0 && ms != nullptr, "bad arguments");
    ms[0] = ms[1] = ms[2] = 0.0;
    if (steps == 0) return NRN_OK;
    for (auto& q : e->projs) {
        if (q.plastic && !q.clamped) {
            NRN_TRY(nrn_cuda_clamp(q.csr.w, q.csr.nnz, static_cast<float>(q.stdp[4]), static_cast<float>(q.stdp[5]),
                                   reinterpret_cast<nrn_stream_t>(e->stream)));
            q.clamped = true;
        }
    }
    cudaEvent_t ev[4];
    for (auto& x : ev) NRN_CUDA_TRY(cudaEventCreate(&x));
    nrn_status_t st = NRN_OK;
    for (int64_t k = 0; k < steps && st == NRN_OK; ++k) {
        st = e->enqueue_step(0, ev);
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
        NRN_CUDA_TRY(cudaStreamSynchronize(e->stream));
        e->step += steps;
    }
    return st;
}

nrn_status_t nrn_engine_set_step(nrn_engine* e, int64_t step) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(step >= 0, "step must be >= 0");
    const long long s = step;
    NRN_CUDA_TRY(cudaMemcpyAsync(e->d_step, &s, sizeof(s), cudaMemcpyHostToDevice, e->stream));
    NRN_CUDA_TRY(cudaStreamSynchronize(e->stream));
    e->step = step;
    return NRN_OK;
}

nrn_status_t nrn_engine_sync(nrn_engine* e) {
    ENGINE_GUARD(e);
    NRN_CUDA_TRY(cudaStreamSynchronize(e->stream));
    return e->check_err();
}

nrn_status_t nrn_engine_raster(nrn_engine* e, int32_t* step, int32_t* gid, int64_t cap, int64_t* n) {
    ENGINE_GUARD(e);
    NRN_CHECK_ARG(n != nullptr, "null count");
    unsigned long long cnt = 0;
    NRN_CUDA_TRY(cudaMemcpyAsync(&cnt, e->d_raster_count, sizeof(cnt), cudaMemcpyDeviceToHost, e->stream));
    NRN_CUDA_TRY(cudaStreamSynchronize(e->stream));
    *n = static_cast<int64_t>(cnt);
    if (cnt == 0) return NRN_OK;
    if (static_cast<int64_t>(cnt) > e->raster_cap)
        return fail(NRN_ERR_CAPACITY, "spike raster overflowed: read it more often (" + std::to_string(cnt) +
                                          " spikes, capacity " + std::to_string(e->raster_cap) + ")");
    if (static_cast<int64_t>(cnt) > cap) return fail(NRN_ERR_CAPACITY, "output buffer too small for the raster");
    // order of the reference's recorder: by step, ascending ids within a step
    NRN_TRY(sort_raster(e->raster_step, e->raster_gid, static_cast<int64_t>(cnt), e->stream));
    NRN_CUDA_TRY(cudaMemcpyAsync(step, e->raster_step, cnt * 4, cudaMemcpyDeviceToHost, e->stream));
    NRN_CUDA_TRY(cudaMemcpyAsync(gid, e->raster_gid, cnt * 4, cudaMemcpyDeviceToHost, e->stream));
    NRN_CUDA_TRY(cudaMemsetAsync(e->d_raster_count, 0, sizeof(unsigned long long), e->stream));
    NRN_CUDA_TRY(cudaStreamSynchronize(e->stream));
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
    NRN_TRY(e->flush_deferred());
    NRN_TRY(e->check_err());
    std::vector<float> w(static_cast<size_t>(c.nnz));
    NRN_CUDA_TRY(cudaStreamSynchronize(e->stream));
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
    NRN_TRY(e->flush_deferred());
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
    unsigned long long ev = 0, rc = 0;
    NRN_CUDA_TRY(cudaMemcpyAsync(&ev, e->d_events, sizeof(ev), cudaMemcpyDeviceToHost, e->stream));
    NRN_CUDA_TRY(cudaMemcpyAsync(&rc, e->d_raster_count, sizeof(rc), cudaMemcpyDeviceToHost, e->stream));
    NRN_CUDA_TRY(cudaStreamSynchronize(e->stream));
    if (events) *events = static_cast<int64_t>(ev);
    if (spikes) *spikes = e->spikes_flushed + static_cast<int64_t>(rc);
    return NRN_OK;
}

}  // extern "C"
