// plastic.cu -- pair STDP with the potentiation deferred to row passes.
//
// The reference's rule (src/plasticity/stdp.cpp:43-141), applied every step
// (slow_ratio 1), changes a weight when its source spikes (-A- x_post, plus
// +A+ x_pre if the target spiked in the same step) or when its target spikes
// (+A+ x_pre).  Applying the target-spike term immediately means one random
// read-modify-write per synapse of every spiking target, the slowest memory
// operation a GPU has.  Here that term is deferred: each (source, delay)
// segment of the source-major CSR records the step T through which its
// weights are up to date, and whenever the segment is walked -- at delivery
// of one of its source's spikes, at the source's own spike, or by a rolling
// sweep that reaches every row once per ~1000 steps -- the potentiations of
// every target spike in (T, now] are replayed first, oldest first, with the
// same float operations in the same order as the immediate update.  The
// weights are therefore the same, bit for bit, as applying the rule every
// step, but every weight access is a contiguous row access.
//
// What the replay needs:
//   * the target's spike steps after T: the last four are kept in one int4
//     per target (L2-resident), older ones in a ring of post_ring_k steps;
//   * x_pre of the source at each of those steps: the neuron update copies
//     x_pre to a snapshot every `period` steps; x_pre(t) is the latest
//     snapshot at or before t (or the value stored at T, if later) multiplied
//     by the decay once per step in between -- the same sequence of float
//     multiplications as the step-by-step trace, as the source does not
//     spike between T and the pass.
// A target that spiked more often than the ring holds, or a snapshot that
// was overwritten, sets the error flag (the sweep keeps both from happening
// for firing rates below ~1 kHz).
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace nrn {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxReplay = 32;

__device__ __forceinline__ float clampw(float w, float lo, float hi) { return fminf(fmaxf(w, lo), hi); }

// x_pre of source j at step t, T < t, no spike of j in (T, t].
__device__ __forceinline__ float x_at(const PlasticArgs& a, int j, int t, int T, float xT) {
    const int s_star = ((t + 1) / a.snap_period) * a.snap_period - 1;
    float x;
    int base;
    if (s_star > T) {
        x = a.x_snap[static_cast<long long>(((s_star + 1) / a.snap_period) % a.snap_depth) * a.n_src + j];
        base = s_star;
    } else {
        x = xT;
        base = T;
    }
    for (int u = base + 1; u <= t; ++u) x = x * a.decay_pre;
    return x;
}

// Potentiation of one synapse for the target spikes in (T, end], oldest first.
__device__ __forceinline__ float replay(const PlasticArgs& a, int j, uint32_t i, int T, float xT, int end, float w,
                                        float mod) {
    const int4 r = a.post_recent[i];
    if (r.x <= T) return w;   // no target spike since T (the common case)
    int steps[kMaxReplay];
    int n = 0;
    const int cand[4] = {r.x, r.y, r.z, r.w};
    bool more = true;
    for (int q = 0; q < 4; ++q) {
        if (cand[q] <= T) { more = false; break; }
        if (cand[q] <= end) steps[n++] = cand[q];
    }
    if (more) {
        // older spikes from the ring (entries cnt-5, cnt-6, ...)
        const int cnt = a.post_cnt[i];
        int idx = cnt - 5;
        const int oldest = cnt - a.post_ring_k;
        for (; idx >= 0; --idx) {
            if (idx < oldest || n >= kMaxReplay) {
                atomicExch(a.err, 1);   // history too short for this gap
                break;
            }
            const int t = a.post_ring[static_cast<long long>(i) * a.post_ring_k + (idx % a.post_ring_k)];
            if (t <= T) break;
            if (t <= end) steps[n++] = t;
        }
    }
    for (int q = n - 1; q >= 0; --q) {
        const float x = x_at(a, j, steps[q], T, xT);
        const float dw = a.a_plus * x;   // (A+ x_pre) * post(=1) - (A- x_post) * pre(=0)
        float upd = (dw * a.lr) * 1.0f;
        if (a.mod) upd = upd * mod;
        w = clampw(w + upd, a.w_min, a.w_max);
    }
    return w;
}

// One segment (source j, delay index k) walked by the whole block.
__device__ void walk_segment(const PlasticArgs& a, int mode, int j, int k, long long step) {
    __shared__ int sh_T;
    __shared__ float sh_xT;
    const long long seg = static_cast<long long>(j) * a.nd + k;
    if (threadIdx.x == 0) {
        sh_T = a.seg_last[seg];
        sh_xT = a.seg_x[seg];
    }
    __syncthreads();
    const int T = sh_T;
    const float xT = sh_xT;
    // Pending potentiation through `end`; the delivery runs before this
    // step's update (end = step - 1), the source-spike update and the sweep
    // after it (the source-spike step itself is handled below).
    const int now = static_cast<int>(step);
    const int end = mode == PLASTIC_FLUSH ? now : now - 1;
    const long long s0 = a.seg_ptr[seg], s1 = a.seg_ptr[seg + 1];
    if (threadIdx.x == 0 && T < now - (a.snap_depth - 1) * a.snap_period)
        atomicExch(a.err, 2);   // segment not visited within the snapshot window
    const float ltp_now = a.a_plus * a.x_pre[j];
    unsigned long long events = 0;
    for (long long syn = s0 + threadIdx.x; syn < s1; syn += kThreads) {
        const uint32_t i = a.tgt[syn];
        const float mod = a.mod ? a.mod[syn] : 1.0f;
        const float w0 = a.w[syn];
        float w = T < end ? replay(a, j, i, T, xT, end, w0, mod) : w0;
        if (mode == PLASTIC_LTD) {
            // the source spiked now: -A- x_post, plus +A+ x_pre if the target did too
            const float dw = ltp_now * a.spike_tgt[i] - (a.a_minus * a.x_post[i]) * 1.0f;
            float upd = (dw * a.lr) * 1.0f;
            if (a.mod) upd = upd * mod;
            w = clampw(w + upd, a.w_min, a.w_max);
        }
        if (__float_as_uint(w) != __float_as_uint(w0)) a.w[syn] = w;
        if (mode == PLASTIC_DELIVER) {
            atomicAdd(a.acc + i, a.mod ? w * mod : w);
            ++events;
        }
    }
    if (mode == PLASTIC_DELIVER && a.events) {
        __shared__ unsigned long long sh_ev;
        if (threadIdx.x == 0) sh_ev = 0;
        __syncthreads();
        if (events) atomicAdd(&sh_ev, events);
        __syncthreads();
        if (threadIdx.x == 0 && sh_ev) atomicAdd(a.events, sh_ev);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        a.seg_last[seg] = mode == PLASTIC_DELIVER ? now - 1 : now;
        a.seg_x[seg] = a.x_pre[j];   // x_pre at the new T (the trace as it is now)
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads) plastic_rows_kernel(const __grid_constant__ PlasticArgs a, int mode,
                                                                long long step_off, const long long* step_base) {
    const long long step = step_off + (step_base ? *step_base : 0);
    __shared__ long long pre[257];
    __shared__ int slots[256];
    long long n_items = 0;
    if (mode == PLASTIC_DELIVER) {
        // spikes of step - (dmin + k) through the delay-k segments
        if (threadIdx.x == 0) {
            long long acc = 0;
            for (int k = 0; k < a.nd; ++k) {
                pre[k] = acc;
                const long long src_step = step - (a.dmin + k);
                slots[k] = src_step >= 0 ? static_cast<int>(src_step % a.hist_src.depth) : -1;
                if (src_step >= 0) acc += a.hist_src.count[slots[k]];
            }
            pre[a.nd] = acc;
        }
        __syncthreads();
        n_items = pre[a.nd];
    } else {
        const int slot = static_cast<int>(step % a.hist_src.depth);
        const long long n_spk = mode == PLASTIC_LTD ? a.hist_src.count[slot] : 0;
        const long long r0 = static_cast<long long>(step % a.sweep_period) * a.sweep_rows;
        const long long left = a.n_src - r0;
        const long long n_sweep = left <= 0 ? 0 : (a.sweep_rows < left ? a.sweep_rows : left);
        n_items = n_spk + (mode == PLASTIC_LTD ? n_sweep : a.n_src);
        for (long long it = blockIdx.x; it < n_items; it += gridDim.x) {
            if (mode == PLASTIC_LTD && it < n_spk) {
                const int j = a.hist_src.ids[static_cast<long long>(slot) * a.hist_src.cap + it];
                for (int k = 0; k < a.nd; ++k) walk_segment(a, PLASTIC_LTD, j, k, step);
            } else {
                const long long r = mode == PLASTIC_LTD ? r0 + (it - n_spk) : it;
                const int j = static_cast<int>(r);
                // a row whose source spiked this step was just updated above
                if (mode == PLASTIC_LTD && a.spike_src[j] != 0.0f) continue;
                for (int k = 0; k < a.nd; ++k) walk_segment(a, PLASTIC_FLUSH, j, k, step);
            }
        }
        return;
    }
    for (long long it = blockIdx.x; it < n_items; it += gridDim.x) {
        int k = 0;
        while (k + 1 < a.nd && pre[k + 1] <= it) ++k;
        const int j = a.hist_src.ids[static_cast<long long>(slots[k]) * a.hist_src.cap + (it - pre[k])];
        walk_segment(a, PLASTIC_DELIVER, j, k, step);
    }
}

}  // namespace

nrn_status_t plastic_rows(const PlasticArgs& a, int mode, long long step_off, const long long* step_base,
                          cudaStream_t s) {
    NRN_CHECK_ARG(a.nd >= 1 && a.nd <= 256, "plastic projection: at most 256 delay values");
    int per_sm = 0;
    NRN_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, plastic_rows_kernel, kThreads, 0));
    const int blocks = std::max(1, per_sm) * sm_count_current();
    plastic_rows_kernel<<<blocks, kThreads, 0, s>>>(a, mode, step_off, step_base);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

}  // namespace nrn
