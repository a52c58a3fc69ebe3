// deliver.cu -- event-driven spike delivery and pair STDP.
//
// Delivery (the reference's phase 2, src/simulation/runner.cpp:106-124, and
// connection_deliver, src/connectivity/connect.cpp:36-79): at step t, every
// projection adds, for each delay d, the weights of the delay-d synapses of
// the neurons that spiked at step t - d into the target accumulator.  The
// reference multiplies the whole (masked) block-dense weight matrix by the
// dense spike vector; here only the synapses of spiking neurons are touched:
// the source-major CSR is segmented by delay, one warp walks one (spike,
// delay) segment, and each synapse is one fire-and-forget float reduction
// (RED.ADD.F32) into the accumulator, which stays resident in L2.
//
// Bytes per delivered synaptic event: 4 (target) + 4 (weight) read,
// 4 reduced into L2; 16 per spike and delay for the two segment offsets.
//
// STDP (src/plasticity/stdp.cpp:43-141): the reference keeps a trace per
// synapse, but every row (column) of its trace blocks receives the same
// decay and increments, so one trace per source (target) neuron is exact.
// A weight changes only when its source or target spiked at this step, so
// the update walks the out-synapses of the spiking sources (LTD term, plus
// LTP when the target spiked too) and the in-synapses of the spiking
// targets whose source did not spike (LTP term); no synapse is visited
// twice, so no atomics are needed.  The per-step clamp of every weight in
// the reference reduces to one clamp of all weights before the first update.
#include <cuda_runtime.h>

#include <algorithm>

#include <cub/block/block_scan.cuh>

#include "common.cuh"
#include "internal.h"

namespace nrn {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxPairs = 1024;   // (projection, delay) pairs per launch
constexpr int kChunk = 128;       // synapses per warp work unit of the STDP kernels (4 per lane)
constexpr int kDeliverVec = 4;    // synapses per lane of one delivery unit
constexpr int kDeliverChunk = 32 * kDeliverVec;
constexpr int kInFlight = 2;      // delivery units whose loads are in flight together

struct DeliverParams {
    nrn_proj_t proj[NRN_MAX_PROJ];
    nrn_spike_hist_t hist[NRN_MAX_POPS];
    int nproj;
    int nhist;
    int npairs;
    int pad;
    long long step_off;
    const long long* step_base;
    unsigned long long* events;
};

// Dynamic shared memory: pair table of npairs entries.
struct PairView {
    long long* start;   // [npairs + 1] exclusive prefix of work units
    int* slot;          // [npairs]
    int* chunks;        // [npairs] units per spike (ceil(max segment / kDeliverChunk))
    short* proj;        // [npairs]
    short* k;           // [npairs]
};

__device__ __forceinline__ PairView pair_view(void* base, int npairs) {
    PairView v;
    v.start = reinterpret_cast<long long*>(base);
    v.slot = reinterpret_cast<int*>(v.start + npairs + 1);
    v.chunks = v.slot + npairs;
    v.proj = reinterpret_cast<short*>(v.chunks + npairs);
    v.k = v.proj + npairs;
    return v;
}

size_t pair_smem(int npairs) {
    return static_cast<size_t>(npairs + 1) * sizeof(long long) + static_cast<size_t>(npairs) * (4 + 4 + 2 + 2) + 16;
}

// Work unit = (spike, delay segment, chunk of kDeliverChunk synapses), one warp
// each.  Every segment of a projection is given ceil(max segment length /
// kDeliverChunk) units (units past the segment's end are empty), so the units of
// one step are numbered without a prefix over segment lengths and spread
// evenly over a full-occupancy grid.
__global__ void __launch_bounds__(kThreads, 5) deliver_kernel(const __grid_constant__ DeliverParams P) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const PairView tab = pair_view(smem_raw, P.npairs);
    using Scan = cub::BlockScan<long long, kThreads>;
    __shared__ typename Scan::TempStorage scan_tmp;
    __shared__ long long carry;

    const long long step = P.step_off + (P.step_base ? *P.step_base : 0);
    if (threadIdx.x == 0) carry = 0;
    if (blockIdx.x == 0 && threadIdx.x < P.nhist) {
        const nrn_spike_hist_t& h = P.hist[threadIdx.x];
        h.count[step % h.depth] = 0;   // this step's slot, filled by the updates that follow
    }
    __syncthreads();

    for (int base = 0; base < P.npairs; base += kThreads) {
        const int pi = base + threadIdx.x;
        long long units = 0;
        if (pi < P.npairs) {
            int q = 0, acc = 0;
            while (q < P.nproj && pi >= acc + P.proj[q].nd) { acc += P.proj[q].nd; ++q; }
            const int k = pi - acc;
            const nrn_proj_t& pr = P.proj[q];
            const long long src_step = step - (pr.dmin + k);
            const int chunks = (pr.max_seg + kDeliverChunk - 1) / kDeliverChunk;
            tab.proj[pi] = static_cast<short>(q);
            tab.k[pi] = static_cast<short>(k);
            tab.chunks[pi] = chunks > 0 ? chunks : 1;
            tab.slot[pi] = 0;
            if (src_step >= 0 && chunks > 0) {
                const nrn_spike_hist_t& h = P.hist[pr.src_hist];
                const int slot = static_cast<int>(src_step % h.depth);
                tab.slot[pi] = slot;
                units = static_cast<long long>(h.count[slot]) * chunks;
            }
        }
        long long excl, total;
        Scan(scan_tmp).ExclusiveSum(units, excl, total);
        if (pi < P.npairs) tab.start[pi] = carry + excl;
        __syncthreads();
        if (threadIdx.x == 0) carry += total;
        __syncthreads();
    }
    if (threadIdx.x == 0) tab.start[P.npairs] = carry;
    __syncthreads();
    const long long n_units = tab.start[P.npairs];

    // Warp w takes units w, w + n_warps, w + 2 n_warps, ...  The lanes first
    // resolve the headers of 32 of them at once (spike id, then segment
    // bounds: two dependent loads, paid once per 32 units), then the warp
    // streams those units kInFlight at a time, the target and weight loads
    // of all of them issued before their reductions.
    const int lane = threadIdx.x & 31;
    const long long warp = (static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const long long n_warps = (static_cast<long long>(gridDim.x) * kThreads) >> 5;
    const long long mine = warp < n_units ? (n_units - warp + n_warps - 1) / n_warps : 0;   // this warp's units
    unsigned long long my_events = 0;
    for (long long hb = 0; hb < mine; hb += 32) {
        const long long u = warp + (hb + lane) * n_warps;
        long long s0 = 0;
        int len = 0, q = 0;
        if (hb + lane < mine) {
            int lo = 0, hi = P.npairs - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (tab.start[mid] <= u) lo = mid; else hi = mid - 1;
            }
            const long long local = u - tab.start[lo];
            const int chunks = tab.chunks[lo];
            const long long spike = local / chunks;
            const int chunk = static_cast<int>(local - spike * chunks);
            q = tab.proj[lo];
            const nrn_proj_t& pr = P.proj[q];
            const nrn_spike_hist_t& h = P.hist[pr.src_hist];
            const int j = h.ids[static_cast<long long>(tab.slot[lo]) * h.cap + spike];
            const long long seg = static_cast<long long>(j) * pr.nd + tab.k[lo];
            const long long e0 = pr.seg_ptr[seg + 1];
            s0 = pr.seg_ptr[seg] + static_cast<long long>(chunk) * kDeliverChunk;
            const long long s1 = s0 + kDeliverChunk < e0 ? s0 + kDeliverChunk : e0;
            len = s1 > s0 ? static_cast<int>(s1 - s0) : 0;
            my_events += static_cast<unsigned long long>(len);
        }
        const int nh = mine - hb < 32 ? static_cast<int>(mine - hb) : 32;
        for (int i = 0; i < nh; i += kInFlight) {
            uint32_t t[kInFlight][kDeliverVec];
            float w[kInFlight][kDeliverVec];
            int n[kInFlight], qa[kInFlight];   // this lane's synapses of the unit: lane + 32 v < n
#pragma unroll
            for (int f = 0; f < kInFlight; ++f) {
                // every lane takes part in the shuffles; units past nh are empty
                const long long a0 = __shfl_sync(0xffffffffu, s0, (i + f) & 31);
                n[f] = __shfl_sync(0xffffffffu, len, (i + f) & 31);
                qa[f] = __shfl_sync(0xffffffffu, q, (i + f) & 31);
                if (i + f >= nh) n[f] = 0;
                const nrn_proj_t& pr = P.proj[qa[f]];
#pragma unroll
                for (int v = 0; v < kDeliverVec; ++v) {
                    if (lane + 32 * v < n[f]) {
                        // the synapse stream is read once a step: evict first, so the
                        // accumulators and spike records stay in L2
                        const long long syn = a0 + lane + 32 * v;
                        t[f][v] = __ldcs(pr.tgt + syn);
                        w[f][v] = __ldcs(pr.w + syn);
                        if (pr.mod != nullptr) w[f][v] = w[f][v] * __ldcs(pr.mod + syn);
                    }
                }
            }
#pragma unroll
            for (int f = 0; f < kInFlight; ++f) {
                float* acc = P.proj[qa[f]].acc;
#pragma unroll
                for (int v = 0; v < kDeliverVec; ++v)
                    if (lane + 32 * v < n[f]) atomicAdd(acc + t[f][v], w[f][v]);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) my_events += __shfl_down_sync(0xffffffffu, my_events, o);
    if (P.events && lane == 0 && my_events) atomicAdd(P.events, my_events);
}

// ---------------------------------------------------------------------------
// STDP
// ---------------------------------------------------------------------------

__device__ __forceinline__ bool stdp_active(const nrn_stdp_t& s, long long step) {
    return s.slow_ratio <= 1 || (step % s.slow_ratio) == 0;
}

__global__ void stdp_trace_kernel(const __grid_constant__ nrn_stdp_t s, long long step_off, const long long* step_base) {
    const long long step = step_off + (step_base ? *step_base : 0);
    if (!stdp_active(s, step)) return;
    const int n_src = s.proj.n_src, n_tgt = s.proj.n_tgt;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_src + n_tgt; i += gridDim.x * blockDim.x) {
        if (i < n_src) s.x_pre[i] = s.x_pre[i] * s.decay_pre + s.spike_src[i];
        else {
            const int k = i - n_src;
            s.x_post[k] = s.x_post[k] * s.decay_post + s.spike_tgt[k];
        }
    }
}

__device__ __forceinline__ float stdp_apply(const nrn_stdp_t& s, long long syn, float w_old, float dw) {
    float upd = (dw * s.lr) * 1.0f;
    if (s.proj.mod) upd = upd * s.proj.mod[syn];
    float w = w_old + upd;
    w = fmaxf(w, s.w_min);
    w = fminf(w, s.w_max);
    return w;
}

// Work units of one warp: (spiking source, chunk of its out-row) -- the
// -A- x_post term, plus +A+ x_pre where the target spiked too -- then
// (spiking target, chunk of its in-list) -- +A+ x_pre where the source did
// not spike.  Chunk counts come from the longest row / in-list.
__global__ void __launch_bounds__(kThreads) stdp_update_kernel(const __grid_constant__ nrn_stdp_t s,
                                                               long long step_off, const long long* step_base) {
    const long long step = step_off + (step_base ? *step_base : 0);
    if (!stdp_active(s, step)) return;
    const int slot_s = static_cast<int>(step % s.hist_src.depth);
    const int slot_t = static_cast<int>(step % s.hist_tgt.depth);
    const int c_pre = s.max_row > 0 ? (s.max_row + kChunk - 1) / kChunk : 1;
    const int c_post = s.max_in > 0 ? (s.max_in + kChunk - 1) / kChunk : 1;
    const long long u_pre = static_cast<long long>(s.hist_src.count[slot_s]) * c_pre;
    const long long n_units = u_pre + static_cast<long long>(s.hist_tgt.count[slot_t]) * c_post;
    const int nd = s.proj.nd;
    const int lane = threadIdx.x & 31;
    const long long warp = (static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const long long n_warps = (static_cast<long long>(gridDim.x) * kThreads) >> 5;
    for (long long u = warp; u < n_units; u += n_warps) {
        if (u < u_pre) {
            const long long it = u / c_pre;
            const int chunk = static_cast<int>(u - it * c_pre);
            const int j = s.hist_src.ids[static_cast<long long>(slot_s) * s.hist_src.cap + it];
            const long long e0 = s.proj.seg_ptr[static_cast<long long>(j + 1) * nd];
            const long long b0 = s.proj.seg_ptr[static_cast<long long>(j) * nd] + static_cast<long long>(chunk) * kChunk;
            const long long b1 = b0 + kChunk < e0 ? b0 + kChunk : e0;
            if (b0 >= b1) continue;
            const float ltp = s.a_plus * s.x_pre[j];
            uint32_t t[4];
            float w[4], post[4], xp[4];
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const long long syn = b0 + lane + 32 * v;
                if (syn < b1) {
                    t[v] = s.proj.tgt[syn];
                    w[v] = s.w_mut[syn];
                }
            }
#pragma unroll
            for (int v = 0; v < 4; ++v)
                if (b0 + lane + 32 * v < b1) {
                    post[v] = s.spike_tgt[t[v]];
                    xp[v] = s.x_post[t[v]];
                }
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const long long syn = b0 + lane + 32 * v;
                if (syn < b1) {
                    const float dw = ltp * post[v] - (s.a_minus * xp[v]) * 1.0f;
                    s.w_mut[syn] = stdp_apply(s, syn, w[v], dw);
                }
            }
        } else {
            const long long it = (u - u_pre) / c_post;
            const int chunk = static_cast<int>((u - u_pre) - it * c_post);
            const int i = s.hist_tgt.ids[static_cast<long long>(slot_t) * s.hist_tgt.cap + it];
            const long long e0 = s.in_ptr[i + 1];
            const long long b0 = s.in_ptr[i] + static_cast<long long>(chunk) * kChunk;
            const long long b1 = b0 + kChunk < e0 ? b0 + kChunk : e0;
            if (b0 >= b1) continue;
            const float ltd = (s.a_minus * s.x_post[i]) * 0.0f;   // the LTD term with pre = 0
            uint32_t j[4];
            long long syn[4];
            float pre[4], xq[4], w[4];
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const long long k = b0 + lane + 32 * v;
                if (k < b1) {
                    j[v] = s.in_src[k];
                    syn[v] = s.in_syn[k];
                }
            }
#pragma unroll
            for (int v = 0; v < 4; ++v)
                if (b0 + lane + 32 * v < b1) {
                    pre[v] = s.spike_src[j[v]];
                    xq[v] = s.x_pre[j[v]];
                    w[v] = s.w_mut[syn[v]];
                }
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                if (b0 + lane + 32 * v < b1 && pre[v] == 0.0f) {   // else handled with the source's row
                    const float dw = (s.a_plus * xq[v]) * 1.0f - ltd;
                    s.w_mut[syn[v]] = stdp_apply(s, syn[v], w[v], dw);
                }
            }
        }
    }
}

__global__ void clamp_kernel(float* w, long long n, float lo, float hi) {
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        w[i] = fminf(fmaxf(w[i], lo), hi);
}

int sm_count() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// Deterministic delivery: one warp per target; the lanes look at 32
// in-synapses at a time (in order), and the weights of those whose source
// spiked are added one by one in that order (a ballot of the hits, then the
// warp walks its set bits), so the sum is the sequential one.
__global__ void __launch_bounds__(256) det_deliver_kernel(const __grid_constant__ DetAcc A, int ring,
                                                         long long step_off, const long long* step_base,
                                                         unsigned long long* events) {
    const long long step = step_off + (step_base ? *step_base : 0);
    const int lane = threadIdx.x & 31;
    const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
    unsigned long long hits = 0;
    for (long long t = warp; t < A.n; t += n_warps) {
        float sum = 0.0f;
        for (int q = 0; q < A.nproj; ++q) {
            const DetProj& P = A.proj[q];
            const long long b = P.ptr[t], e = P.ptr[t + 1];
            for (long long base = b; base < e; base += 32) {
                const long long k = base + lane;
                float v = 0.0f;
                bool hit = false;
                if (k < e) {
                    const int d = P.delay[k];
                    const long long s_src = step - d;
                    if (s_src >= 0) {
                        const uint32_t j = P.src[k];
                        hit = P.flags[static_cast<long long>(s_src % ring) * P.flag_n + j] != 0;
                    }
                    if (hit) {
                        const uint32_t syn = P.syn[k];
                        v = P.w[syn];
                        if (P.mod) v = v * P.mod[syn];
                    }
                }
                unsigned m = __ballot_sync(0xffffffffu, hit);
                hits += __popc(m);
                while (m) {
                    const int l = __ffs(m) - 1;
                    sum = sum + __shfl_sync(0xffffffffu, v, l);
                    m &= m - 1;
                }
            }
        }
        if (lane == 0) A.acc[t] = sum;
    }
    if (events && lane == 0 && hits) atomicAdd(events, hits);
}

__global__ void det_flags_kernel(const float* spike, int n, uint8_t* flags, int ring, long long step_off,
                                 const long long* step_base) {
    const long long step = step_off + (step_base ? *step_base : 0);
    uint8_t* row = flags + static_cast<long long>(step % ring) * n;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        row[i] = spike[i] != 0.0f ? 1 : 0;
}

}  // namespace

nrn_status_t det_deliver(const DetAcc& a, int32_t ring, long long step_off, const long long* step_base,
                         unsigned long long* events, cudaStream_t s) {
    NRN_CHECK_ARG(a.nproj >= 0 && a.nproj <= 8, "deterministic delivery: at most 8 projections per input");
    NRN_CHECK_ARG(ring >= 1, "deterministic delivery: bad flag ring");
    if (a.n == 0) return NRN_OK;
    const int blocks = static_cast<int>(std::min<long long>((static_cast<long long>(a.n) * 32 + 255) / 256,
                                                            32LL * sm_count()));
    det_deliver_kernel<<<blocks, 256, 0, s>>>(a, ring, step_off, step_base, events);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

nrn_status_t det_flags(const float* spike, int32_t n, uint8_t* flags, int32_t ring, long long step_off,
                       const long long* step_base, cudaStream_t s) {
    if (n == 0) return NRN_OK;
    const int blocks = std::min((n + 255) / 256, 8 * sm_count());
    det_flags_kernel<<<blocks, 256, 0, s>>>(spike, n, flags, ring, step_off, step_base);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

}  // namespace nrn

extern "C" nrn_status_t nrn_cuda_deliver(const nrn_proj_t* projs, int32_t nproj, const nrn_spike_hist_t* hists,
                                         int32_t nhist, int64_t step_off, const int64_t* step_base,
                                         nrn_stream_t stream) {
    using namespace nrn;
    return nrn_cuda_deliver_counted(projs, nproj, hists, nhist, step_off, step_base, nullptr, stream);
}

extern "C" nrn_status_t nrn_cuda_deliver_counted(const nrn_proj_t* projs, int32_t nproj,
                                                 const nrn_spike_hist_t* hists, int32_t nhist,
                                                 int64_t step_off, const int64_t* step_base,
                                                 unsigned long long* events, nrn_stream_t stream) {
    using namespace nrn;
    NRN_CHECK_ARG(nproj >= 0 && nproj <= NRN_MAX_PROJ, "nrn_cuda_deliver: too many projections");
    NRN_CHECK_ARG(nhist >= 0 && nhist <= NRN_MAX_POPS, "nrn_cuda_deliver: too many populations");
    NRN_CHECK_ARG(nproj == 0 || projs != nullptr, "nrn_cuda_deliver: null projections");
    NRN_CHECK_ARG(nhist == 0 || hists != nullptr, "nrn_cuda_deliver: null histories");
    DeliverParams P{};
    int pairs = 0;
    for (int q = 0; q < nproj; ++q) {
        const nrn_proj_t& p = projs[q];
        NRN_CHECK_ARG(p.dmin >= 1 && p.nd >= 1, "nrn_cuda_deliver: delays must be >= 1 step");
        NRN_CHECK_ARG(p.src_hist >= 0 && p.src_hist < nhist, "nrn_cuda_deliver: bad source history");
        NRN_CHECK_ARG(p.dmin + p.nd - 1 < hists[p.src_hist].depth,
                      "nrn_cuda_deliver: history shallower than the longest delay");
        NRN_CHECK_ARG(p.seg_ptr && p.tgt && p.w && p.acc, "nrn_cuda_deliver: null projection array");
        P.proj[q] = p;
        pairs += p.nd;
    }
    NRN_CHECK_ARG(pairs <= kMaxPairs, "nrn_cuda_deliver: too many (projection, delay) pairs");
    for (int h = 0; h < nhist; ++h) {
        NRN_CHECK_ARG(hists[h].depth >= 1 && hists[h].ids && hists[h].count, "nrn_cuda_deliver: bad history");
        P.hist[h] = hists[h];
    }
    P.nproj = nproj;
    P.nhist = nhist;
    P.npairs = pairs;
    P.step_off = step_off;
    P.step_base = reinterpret_cast<const long long*>(step_base);
    P.events = events;
    const size_t smem = pair_smem(pairs);
    int per_sm = 0;
    NRN_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, deliver_kernel, kThreads, smem));
    const int blocks = std::max(1, per_sm) * sm_count();   // one full wave
    deliver_kernel<<<blocks, kThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(P);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

extern "C" nrn_status_t nrn_cuda_stdp_step(const nrn_stdp_t* s, int64_t step_off, const int64_t* step_base,
                                           nrn_stream_t stream) {
    using namespace nrn;
    NRN_CHECK_ARG(s != nullptr, "nrn_cuda_stdp_step: null arguments");
    NRN_CHECK_ARG(s->w_mut && s->in_ptr && s->in_syn && s->in_src && s->x_pre && s->x_post && s->spike_src &&
                      s->spike_tgt && s->proj.seg_ptr && s->proj.tgt,
                  "nrn_cuda_stdp_step: null array");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int n = s->proj.n_src + s->proj.n_tgt;
    const int tb = 256;
    const int trace_blocks = std::max(1, std::min((n + tb - 1) / tb, 8 * sm_count()));
    const long long* base = reinterpret_cast<const long long*>(step_base);
    if (!s->traces_updated) {
        stdp_trace_kernel<<<trace_blocks, tb, 0, st>>>(*s, step_off, base);
        NRN_CUDA_TRY(cudaGetLastError());
    }
    int per_sm = 0;
    NRN_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, stdp_update_kernel, kThreads, 0));
    stdp_update_kernel<<<std::max(1, per_sm) * sm_count(), kThreads, 0, st>>>(*s, step_off, base);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

extern "C" nrn_status_t nrn_cuda_clamp(float* w, int64_t n, float lo, float hi, nrn_stream_t stream) {
    using namespace nrn;
    NRN_CHECK_ARG(n >= 0 && (n == 0 || w != nullptr), "nrn_cuda_clamp: bad arguments");
    if (n == 0) return NRN_OK;
    const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 16 * sm_count()));
    clamp_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(w, n, lo, hi);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}
