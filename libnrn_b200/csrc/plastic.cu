// plastic.cu -- pair STDP applied by walks over (source, delay) segments.
//
// The reference's rule (src/plasticity/stdp.cpp:43-141), applied at every
// step (slow_ratio 1), changes a weight at each step where its source or its
// target spiked:
//     dw = (A+ x_pre) * post - (A- x_post) * pre,   w <- clamp(w + dw*lr*mod)
// with x_pre, x_post the traces after this step's decay and increment.  A
// synapse's weight is read only when one of its source's spikes is
// delivered through it, so its updates need not be applied when they
// happen: each (source, delay) segment of the source-major CSR records the
// step T through which its weights are up to date, and a walk of the
// segment applies, synapse by synapse and in time order, the updates of
// every source or target spike in (T, end] -- the same float operations in
// the same order as updating at every step, hence the same weights bit for
// bit.  Walks happen
//   * when a spike arrives through the segment (end = the previous step),
//     followed by the delivery of the updated weight: one contiguous pass
//     over the segment per delivered spike, no random read-modify-write;
//   * in a rolling sweep that looks at every row once per sweep_period
//     steps and walks the segments not walked for `stale` steps, so the
//     spike histories and trace snapshots a walk reads stay short;
//   * over all segments before weights are read (flush).
//
// The traces at a past step t are rebuilt from snapshots: the trace value at
// the end of every window of `win` steps is kept (exchange.cu), and x(t) is
// that value advanced step by step -- x <- x*decay + spike -- through t,
// the same operations as the per-step update.  A walk needs the spike steps
// of the source (newest four per neuron, older ones in a ring for the
// neurons of this GPU) and of each target.
//
// Work unit: one warp per (arriving spike, segment chunk of `chunk` synapses);
// the last chunk of a segment to finish advances the segment's T.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>

#include <cub/block/block_scan.cuh>

#include "common.cuh"
#include "internal.h"

namespace nrn {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxPost = 64;     // target spike steps one walk may need (the ring depth)
constexpr int kMaxPre = 8;       // source spike steps one walk may need
constexpr int kMaxSpan = 1280;   // steps one walk may cover (x_pre table per warp)

enum { ERR_HISTORY = 1, ERR_SNAPSHOT = 2 };

__device__ __forceinline__ void set_err(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ float clampw(float w, float lo, float hi) { return fminf(fmaxf(w, lo), hi); }

// Ascending spike steps: up to four in registers (the common case) ...
struct Steps4 {
    int v0 = 0, v1 = 0, v2 = 0, v3 = 0;
    int n = 0;
    __device__ __forceinline__ int operator[](int k) const { return k == 0 ? v0 : k == 1 ? v1 : k == 2 ? v2 : v3; }
    __device__ __forceinline__ void push(int t) {
        v0 = n == 0 ? t : v0;
        v1 = n == 1 ? t : v1;
        v2 = n == 2 ? t : v2;
        v3 = n == 3 ? t : v3;
        ++n;
    }
};
// ... or in memory (shared, or local for long histories).
struct StepsPtr {
    const int* p = nullptr;
    int n = 0;
    __device__ __forceinline__ int operator[](int k) const { return p[k]; }
};

// The steps in (lo, hi] of a newest-first int4 that holds all of them (its
// oldest entry is at or before lo), ascending.
__device__ __forceinline__ Steps4 steps_from4(int4 r, int lo, int hi) {
    Steps4 s;
    if (r.w > lo && r.w <= hi) s.push(r.w);
    if (r.z > lo && r.z <= hi) s.push(r.z);
    if (r.y > lo && r.y <= hi) s.push(r.y);
    if (r.x > lo && r.x <= hi) s.push(r.x);
    return s;
}

// Spike steps of neuron `idx` in (lo, hi], ascending, into out[0..cap).
// r: newest four steps (newest first, -1 = none); ring/cnt: all steps, if
// kept for this neuron.  Returns the count, or -1 if the kept history does
// not reach back to lo or holds more than cap steps in the range.
__device__ int spikes_in(int4 r, const int32_t* ring, const int32_t* cnt, long long idx, int ring_k, int lo, int hi,
                         int* out, int cap) {
    int n = 0;
    const int c4[4] = {r.x, r.y, r.z, r.w};
    bool more = true;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int t = c4[q];
        if (!more || t <= lo) {
            more = false;
            continue;
        }
        if (t <= hi) {
            if (n == cap) return -1;
            out[n++] = t;
        }
    }
    if (more) {
        // all four newest steps are after lo: older ones from the ring
        if (ring == nullptr) return -1;
        const int c = cnt[idx];
        const int oldest = c - ring_k;
        for (int e = c - 5; e >= 0; --e) {
            if (e < oldest) return -1;
            const int t = ring[idx * ring_k + (e % ring_k)];
            if (t <= lo) break;
            if (t <= hi) {
                if (n == cap) return -1;
                out[n++] = t;
            }
        }
    }
    for (int q = 0; q < n / 2; ++q) {
        const int x = out[q];
        out[q] = out[n - 1 - q];
        out[n - 1 - q] = x;
    }
    return n;
}

struct Seg {
    int j;            // source
    long long seg;    // j * nd + k
    uint32_t s0, s1;  // synapse range (a projection holds < 2^32 synapses)
    int T;            // events applied through T
    int e;            // apply through e
    StepsPtr P;       // source spikes in (T, e] (per-warp shared memory)
    const float* X;   // x_pre(T + 1 + u) at X[u], u < e - T (per-warp shared memory)
};

// Target trace at source spike t (xp0: already loaded for the first one).
__device__ __forceinline__ float x_post_at(const WalkArgs& a, const Seg& g, uint32_t i, int t, int now, float xp0) {
    if (t == g.P[0]) return xp0;
    if (now - t >= a.post_depth) set_err(a.err, ERR_SNAPSHOT);
    return a.post_ring[static_cast<long long>(t & (a.post_depth - 1)) * a.n_tgt + i];
}

// One synapse: every update in (T, e], oldest first.
template <bool MOD, class L>
__device__ __forceinline__ float apply_events(const WalkArgs& a, const Seg& g, const L& Q, uint32_t i, float w,
                                              float mod, int now, float xp0) {
    int p = 0, q = 0;
    while (p < g.P.n || q < Q.n) {
        const int tp = p < g.P.n ? g.P[p] : INT_MAX;
        const int tq = q < Q.n ? Q[q] : INT_MAX;
        const int t = tp < tq ? tp : tq;
        const bool pre = tp == t, post = tq == t;
        const float xpre = post ? g.X[t - g.T - 1] : 0.0f;
        const float xpost = pre ? x_post_at(a, g, i, t, now, xp0) : 0.0f;
        const float dw = (a.a_plus * xpre) * (post ? 1.0f : 0.0f) - (a.a_minus * xpost) * (pre ? 1.0f : 0.0f);
        float upd = (dw * a.lr) * 1.0f;
        if (MOD) upd = upd * mod;
        w = clampw(w + upd, a.w_min, a.w_max);
        if (pre) ++p;
        if (post) ++q;
    }
    return w;
}

template <bool MOD>
__device__ __noinline__ float walk_syn_long(const WalkArgs& a, const Seg& g, uint32_t i, int4 r, float w, float mod,
                                            int now, float xp0) {
    int buf[kMaxPost];
    StepsPtr Q;
    Q.p = buf;
    Q.n = spikes_in(r, a.tgt_ring, a.tgt_cnt, i, a.ring_k, g.T, g.e, buf, kMaxPost);
    if (Q.n < 0) {
        set_err(a.err, ERR_HISTORY);
        return w;
    }
    return apply_events<MOD>(a, g, Q, i, w, mod, now, xp0);
}

// w after one update of the reference's rule with the given spike flags and
// traces (stdp.cpp:130-139): dw = (A+ x_pre) post - (A- x_post) pre.
template <bool MOD>
__device__ __forceinline__ float stdp_apply1(const WalkArgs& a, float w, float mod, float xpre, float post, float xpost,
                                             float pre) {
    const float dw = (a.a_plus * xpre) * post - (a.a_minus * xpost) * pre;
    float upd = (dw * a.lr) * 1.0f;
    if (MOD) upd = upd * mod;
    return clampw(w + upd, a.w_min, a.w_max);
}

// Potentiation by a target spike alone: the general update with post = 1,
// pre = 0.  With finite parameters (nrn_engine_set_stdp checks) the LTD term
// (A- * 0) * 0 is +0 and the update reduces to clamp(w + (A+ x_pre) * lr).
template <bool MOD>
__device__ __forceinline__ float stdp_ltp(const WalkArgs& a, float w, float mod, float xpre) {
    float upd = (a.a_plus * xpre) * a.lr;
    if (MOD) upd = upd * mod;
    return clampw(w + upd, a.w_min, a.w_max);
}

// The common case, straight-line: one source spike t1 in (T, e] and the
// target's spikes in (T, e] among its newest four (r, newest first).
// Target spikes before t1, then t1 (with the target's own spike at t1 if
// any), then target spikes after t1 -- the order of apply_events.
template <bool MOD>
__device__ __forceinline__ float walk_one_pre(const WalkArgs& a, const Seg& g, int t1, int4 r, float w, float mod,
                                              float xp0) {
    const int q4[4] = {r.w, r.z, r.y, r.x};   // oldest first
    const float* X = g.X - (g.T + 1);         // X[t] = x_pre(t)
    bool coincide = false;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int q = q4[k];
        if (q > g.T && q < t1) w = stdp_ltp<MOD>(a, w, mod, X[q]);
        coincide = coincide || q == t1;
    }
    w = stdp_apply1<MOD>(a, w, mod, coincide ? X[t1] : 0.0f, coincide ? 1.0f : 0.0f, xp0, 1.0f);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int q = q4[k];
        if (q > t1 && q <= g.e) w = stdp_ltp<MOD>(a, w, mod, X[q]);
    }
    return w;
}

template <bool MOD>
__device__ __forceinline__ float walk_syn(const WalkArgs& a, const Seg& g, int t1, uint32_t i, int4 r, float w,
                                          float mod, int now, float xp0) {
    if (g.P.n == 1 && r.w <= g.T) return walk_one_pre<MOD>(a, g, t1, r, w, mod, xp0);
    if (g.P.n == 0 && r.x <= g.T) return w;   // nothing happened to this synapse
    if (r.w <= g.T) return apply_events<MOD>(a, g, steps_from4(r, g.T, g.e), i, w, mod, now, xp0);
    return walk_syn_long<MOD>(a, g, i, r, w, mod, now, xp0);
}

// The source trace over (T, e] into the warp's shared table, window by
// window (one window per lane) from the snapshot at the window's start --
// or, for the first, from x_pre(T) -- with the same operations as the
// per-step update.
__device__ __forceinline__ void build_table(const WalkArgs& a, const Seg& g, float* sX, float xT, int m_new,
                                            int lane) {
    const int W = a.win, e = g.e;
    const int m0 = (g.T + 1) / W + 1;   // window ends b = m*W - 1 in (T, e): m = m0, m0+1, ...
    const int n_pieces = 1 + (m0 * W - 1 < e ? (e - (m0 * W - 1) + W - 1) / W : 0);
    for (int pc = lane; pc < n_pieces; pc += 32) {
        int start;
        float x;
        if (pc == 0) {
            start = g.T;
            x = xT;
        } else {
            const int m = m0 + pc - 1;
            start = m * W - 1;
            if (m_new - m >= a.pre_depth) set_err(a.err, ERR_SNAPSHOT);
            x = a.pre_snap[static_cast<long long>(g.j) * a.pre_depth + (m & (a.pre_depth - 1))];
        }
        const int stop = pc == 0 ? (m0 * W - 1 < e ? m0 * W - 1 : e) : (start + W < e ? start + W : e);
        int q = 0;
        while (q < g.P.n && g.P[q] <= start) ++q;
        int next = q < g.P.n ? g.P[q] : INT_MAX;
        for (int u = start + 1; u <= stop; ++u) {
            float sp = 0.0f;
            if (next == u) {
                sp = 1.0f;
                ++q;
                next = q < g.P.n ? g.P[q] : INT_MAX;
            }
            x = x * a.decay_pre + sp;
            sX[u - g.T - 1] = x;
        }
    }
    __syncwarp();
}

// Walks synapses [c0, c1) of the segment, one per lane and round; with
// deliver, adds the updated weights into the target accumulators.
template <bool MOD>
__device__ __forceinline__ unsigned walk_chunk(const WalkArgs& a, const Seg& g, uint32_t c0, uint32_t c1,
                                               bool deliver, int now, int lane, uint32_t t_first, float w_first) {
    // the target trace at the first source spike is loaded with the target's spike steps
    const bool has_pre = g.P.n > 0;
    const int t0 = has_pre ? g.P[0] : 0;
    if (has_pre && now - t0 >= a.post_depth) set_err(a.err, ERR_SNAPSHOT);
    const float* ring0 = a.post_ring + static_cast<long long>(t0 & (a.post_depth - 1)) * a.n_tgt;
    // the next round's target and weight (the HBM stream) are loaded a round
    // ahead; the target's spike steps and trace (L2) within the round
    unsigned n = 0;
    const uint32_t len = c1 - c0;   // at most one chunk: offsets never wrap
    uint32_t t_next = t_first;
    float w_next = w_first;
#pragma unroll 1
    for (uint32_t o = lane; o < len; o += 32) {
        const uint32_t syn = c0 + o;
        const uint32_t t = t_next;
        const float w = w_next;
        const int4 r = a.tgt_recent[t];
        const float xp0 = has_pre ? ring0[t] : 0.0f;
        const float md = MOD ? __ldcs(a.mod + syn) : 1.0f;
        if (o + 32 < len) {
            t_next = __ldcs(a.tgt + syn + 32);
            w_next = a.w[syn + 32];
        }
        const float w1 = walk_syn<MOD>(a, g, t0, t, r, w, md, now, xp0);
        if (__float_as_uint(w1) != __float_as_uint(w)) a.w[syn] = w1;
        if (deliver) {
            atomicAdd(a.acc + t, MOD ? w1 * md : w1);
            ++n;
        }
    }
    return n;
}

// New segment state after a walk through g.e.
__device__ __forceinline__ void finish_seg(const WalkArgs& a, const Seg& g) {
    a.seg_x[g.seg] = g.X[g.e - g.T - 1];
    a.seg_last[g.seg] = g.e;
}

// One chunk of a.chunk synapses of segment (j, k): applies the updates
// through e (and, with deliver, delivers the updated weights); the last
// chunk of the segment to finish records the segment's new state.  Every
// chunk of a segment reads the same state (the write happens only after
// all of them have counted themselves) and so makes the same decision.
// With sweep, the chunk is skipped when its source has spikes still to
// arrive (their walks come) or the segment was walked recently.  Loads are
// grouped so that the chain per chunk is: segment bounds, state and source
// spike steps (one round trip); trace snapshots and the first synapses
// (one); the targets' spike steps and trace (one).  Returns the number of
// events this lane delivered.
template <bool MOD>
__device__ unsigned segment_chunk(const WalkArgs& a, int* sP, float* sX, int j, int k, int chunk, int e,
                                  bool deliver, bool sweep, int now, int m_new, int lane) {
    __syncwarp();   // the warp is done with the previous segment's lists
    const long long seg = static_cast<long long>(j) * a.nd + k;
    uint32_t s0 = 0, s1 = 0;
    int T = 0;
    float xT = 0.0f;
    int4 rj = make_int4(-1, -1, -1, -1);
    if (lane == 0) {
        s0 = static_cast<uint32_t>(a.seg_ptr[seg]);
        s1 = static_cast<uint32_t>(a.seg_ptr[seg + 1]);
        T = a.seg_last[seg];
        xT = a.seg_x[seg];
        rj = a.src_recent[j];
    }
    s0 = __shfl_sync(0xffffffffu, s0, 0);
    s1 = __shfl_sync(0xffffffffu, s1, 0);
    T = __shfl_sync(0xffffffffu, T, 0);
    if (sweep) {
        const int newest = __shfl_sync(0xffffffffu, rj.x, 0);
        if (newest >= now - (a.dmin + a.nd - 1) || T >= now - a.stale) return 0;
    }
    if (static_cast<uint32_t>(chunk) * static_cast<uint32_t>(a.chunk) >= s1 - s0) return 0;
    const uint32_t c0 = s0 + static_cast<uint32_t>(chunk) * static_cast<uint32_t>(a.chunk);
    const uint32_t c1 = s1 - c0 > static_cast<uint32_t>(a.chunk) ? c0 + a.chunk : s1;
    // the first round's synapses, independent of the segment's history
    uint32_t t_first = 0;
    float w_first = 0.0f;
    if (static_cast<uint32_t>(lane) < c1 - c0) {
        t_first = __ldcs(a.tgt + c0 + lane);
        w_first = a.w[c0 + lane];
    }
    unsigned n = 0;
    int nP = -2;   // -2: nothing to apply (walked through e already)
    if (T < e) {
        nP = -1;
        if (lane == 0) {
            if (e - T > kMaxSpan) {
                set_err(a.err, ERR_SNAPSHOT);
            } else {
                const bool own = j >= a.src_lo && j < a.src_hi;
                nP = spikes_in(rj, own ? a.src_ring : nullptr, a.src_cnt, j - a.src_lo, a.ring_k, T, e, sP, kMaxPre);
                if (nP < 0) set_err(a.err, ERR_HISTORY);
            }
        }
        nP = __shfl_sync(0xffffffffu, nP, 0);
        __syncwarp();
    }
    if (nP >= 0) {
        Seg g;
        g.j = j;
        g.seg = seg;
        g.s0 = s0;
        g.s1 = s1;
        g.T = T;
        g.e = e;
        g.P.p = sP;
        g.P.n = nP;
        g.X = sX;
        build_table(a, g, sX, __shfl_sync(0xffffffffu, xT, 0), m_new, lane);
        n = walk_chunk<MOD>(a, g, c0, c1, deliver, now, lane, t_first, w_first);
        __syncwarp();
        if (lane == 0) {
            const int n_chunks = static_cast<int>((s1 - s0 + a.chunk - 1) / a.chunk);
            __threadfence();
            const int done = atomicAdd(a.seg_done + seg, 1);
            if (done == n_chunks - 1) {
                __threadfence();
                a.seg_done[seg] = 0;
                finish_seg(a, g);
            }
        }
    } else if (deliver) {
        // nothing to apply (or a history error, flagged): deliver only
        const uint32_t len = c1 - c0;
        if (static_cast<uint32_t>(lane) < len) {
            atomicAdd(a.acc + t_first, MOD ? w_first * __ldg(a.mod + c0 + lane) : w_first);
            ++n;
        }
        for (uint32_t o = lane + 32; o < len; o += 32) {
            const uint32_t syn = c0 + o;
            const float wv = a.w[syn];
            atomicAdd(a.acc + __ldg(a.tgt + syn), MOD ? wv * __ldg(a.mod + syn) : wv);
            ++n;
        }
    }
    return n;
}

template <bool MOD>
__global__ void __launch_bounds__(kThreads, 4) walk_kernel(const __grid_constant__ WalkArgs a, int mode,
                                                        long long step_off, const long long* step_base) {
    using Scan = cub::BlockScan<long long, kThreads>;
    __shared__ typename Scan::TempStorage scan_tmp;
    __shared__ long long start[257];
    __shared__ int slot[256];
    __shared__ int sP_all[kWarps][kMaxPre];
    __shared__ float sX_all[kWarps][kMaxSpan];
    int* sP = sP_all[threadIdx.x >> 5];
    float* sX = sX_all[threadIdx.x >> 5];

    const long long step = step_off + (step_base ? *step_base : 0);
    const int now = static_cast<int>(step);
    const int m_new = static_cast<int>(step / a.win);   // newest snapshot written
    const int lane = threadIdx.x & 31;
    const long long warp = (static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const long long n_warps = (static_cast<long long>(gridDim.x) * kThreads) >> 5;

    const int chunks = (a.max_seg + a.chunk - 1) / a.chunk > 0 ? (a.max_seg + a.chunk - 1) / a.chunk : 1;
    const long long per_row = static_cast<long long>(a.nd) * chunks;   // units of one source row

    if (mode == WALK_FLUSH) {
        // every segment through step - 1
        const long long n_units = static_cast<long long>(a.n_src) * per_row;
        for (long long u = warp; u < n_units; u += n_warps) {
            const long long row = u / per_row;
            const int rem = static_cast<int>(u - row * per_row);
            segment_chunk<MOD>(a, sP, sX, static_cast<int>(row), rem / chunks, rem % chunks, now - 1, false, false,
                               now, m_new, lane);
        }
        return;
    }

    // Arrivals: spikes of step - (dmin + k) through the delay-k segments,
    // `chunks` units each.
    long long units = 0;
    if (threadIdx.x < a.nd) {
        const long long src_step = step - (a.dmin + threadIdx.x);
        slot[threadIdx.x] = src_step >= 0 ? static_cast<int>(src_step % a.hist_src.depth) : 0;
        if (src_step >= 0) units = static_cast<long long>(a.hist_src.count[slot[threadIdx.x]]) * chunks;
    }
    long long excl, n_arr;
    Scan(scan_tmp).ExclusiveSum(units, excl, n_arr);
    if (threadIdx.x < a.nd) start[threadIdx.x] = excl;
    if (threadIdx.x == 0) start[a.nd] = n_arr;
    __syncthreads();

    // Sweep: rows [r0, r0 + rows), `chunks` units per segment.
    const long long r0 = (step % a.sweep_period) * a.sweep_rows;
    const long long left = a.n_src - r0;
    const long long rows = left <= 0 ? 0 : (a.sweep_rows < left ? a.sweep_rows : left);
    const long long n_units = n_arr + rows * per_row;
    const int win_end = static_cast<int>((step / a.win) * a.win) - 1;   // spikes of all ranks known through here

    unsigned long long my_events = 0;
    for (long long u = warp; u < n_units; u += n_warps) {
        if (u < n_arr) {
            int lo = 0, hi = a.nd - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (start[mid] <= u) lo = mid; else hi = mid - 1;
            }
            const int k = lo;
            const int local = static_cast<int>(u - start[k]);   // < spikes * chunks of one slot
            const int spike = local / chunks;
            const int chunk = local - spike * chunks;
            const int j = a.hist_src.ids[static_cast<long long>(slot[k]) * a.hist_src.cap + spike];
            my_events += segment_chunk<MOD>(a, sP, sX, j, k, chunk, now - 1, true, false, now, m_new, lane);
        } else {
            const int q = static_cast<int>(u - n_arr);   // < sweep rows * per_row
            const int row = q / static_cast<int>(per_row);
            const int rem = q - row * static_cast<int>(per_row);
            const int j = static_cast<int>(r0 + row);
            const int k = rem / chunks;
            segment_chunk<MOD>(a, sP, sX, j, k, rem % chunks, win_end, false, true, now, m_new, lane);
        }
    }
    // lane sums -> one atomic per warp
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) my_events += __shfl_down_sync(0xffffffffu, my_events, o);
    if (a.events && lane == 0 && my_events) atomicAdd(a.events, my_events);
}

}  // namespace

nrn_status_t walk_launch(const WalkArgs& a, int mode, long long step_off, const long long* step_base,
                         cudaStream_t s) {
    NRN_CHECK_ARG(a.nd >= 1 && a.nd <= 256, "plastic projection: at most 256 delay values");
    NRN_CHECK_ARG(a.win >= 1 && a.sweep_period >= 1, "plastic projection: bad window or sweep period");
    NRN_CHECK_ARG(a.chunk >= 32 && a.chunk % 32 == 0, "plastic projection: chunk must be a multiple of 32");
    NRN_CHECK_ARG(a.pre_depth > 0 && (a.pre_depth & (a.pre_depth - 1)) == 0 && a.post_depth > 0 &&
                      (a.post_depth & (a.post_depth - 1)) == 0,
                  "plastic projection: trace ring depths must be powers of two");
    int per_sm = 0;
    if (a.mod) {
        NRN_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, walk_kernel<true>, kThreads, 0));
        walk_kernel<true><<<std::max(1, per_sm) * sm_count_current(), kThreads, 0, s>>>(a, mode, step_off, step_base);
    } else {
        NRN_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, walk_kernel<false>, kThreads, 0));
        walk_kernel<false><<<std::max(1, per_sm) * sm_count_current(), kThreads, 0, s>>>(a, mode, step_off, step_base);
    }
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

}  // namespace nrn
