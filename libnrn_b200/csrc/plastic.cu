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
// Work unit: one block per (arriving spike, segment), its threads striding
// over the segment's synapses, sharing the segment's source spike steps and
// trace table; sweep and flush units look at groups of segments and walk
// those that need it.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>

#include <cub/block/block_scan.cuh>

#include "common.cuh"
#include "internal.h"

namespace nrn {
namespace {

constexpr int kThreads = 256;
constexpr int kMinBlocks = 4;    // 64 registers a thread
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

// The source trace over (T, e] into the block's shared table, window by
// window (one window per thread) from the snapshot at the window's start --
// or, for the first, from x_pre(T) -- with the same operations as the
// per-step update.
__device__ __forceinline__ void build_table(const WalkArgs& a, const Seg& g, float* sX, float xT, int m_new,
                                            int tid) {
    const int W = a.win, e = g.e;
    const int m0 = (g.T + 1) / W + 1;   // window ends b = m*W - 1 in (T, e): m = m0, m0+1, ...
    const int n_pieces = 1 + (m0 * W - 1 < e ? (e - (m0 * W - 1) + W - 1) / W : 0);
    for (int pc = tid; pc < n_pieces; pc += kThreads) {
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
}

// Walks the segment's synapses, thread tid taking offsets tid, tid +
// kThreads, ...; with deliver, adds the updated weights into the target
// accumulators.
template <bool MOD>
__device__ __forceinline__ unsigned walk_block(const WalkArgs& a, const Seg& g, bool deliver, int now, int tid,
                                               uint32_t t_first, float w_first) {
    // the target trace at the first source spike is loaded with the target's spike steps
    const bool has_pre = g.P.n > 0;
    const int t0 = has_pre ? g.P[0] : 0;
    if (has_pre && now - t0 >= a.post_depth) set_err(a.err, ERR_SNAPSHOT);
    const float* ring0 = a.post_ring + static_cast<long long>(t0 & (a.post_depth - 1)) * a.n_tgt;
    // the next round's target and weight (the HBM stream) are loaded a round
    // ahead; the target's spike steps and trace (L2) within the round
    unsigned n = 0;
    const uint32_t len = g.s1 - g.s0;   // a projection holds < 2^32 synapses
    uint32_t t_next = t_first;
    float w_next = w_first;
#pragma unroll 1
    for (uint32_t o = tid; o < len; o += kThreads) {
        const uint32_t syn = g.s0 + o;
        const uint32_t t = t_next;
        const float w = w_next;
        const int4 r = a.tgt_recent[t];
        const float xp0 = has_pre ? ring0[t] : 0.0f;
        const float md = MOD ? __ldcs(a.mod + syn) : 1.0f;
        if (o + kThreads < len) {
            t_next = __ldcs(a.tgt + syn + kThreads);
            w_next = a.w[syn + kThreads];
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

// The segment state one block reads before walking (thread 0 loads it).
struct SegHead {
    uint32_t s0, s1;
    int T;
    int nP;   // source spikes in (T, e]; -2: walked through e already; -1: history error (flagged)
    float xT;
};

// Segment (j, k) by the whole block: applies the updates through e and,
// with deliver, delivers the updated weights.  The load chain is: segment
// bounds, state and source spike steps (thread 0, one round trip); trace
// snapshots and the first synapses (one); the targets' spike steps and
// trace (one per round).  A segment is walked by one block at a time (an
// arrival walk and a sweep walk never meet: the sweep skips sources with
// spikes still to arrive), so the block records the new state as soon as
// its trace table is built.  Returns the number of events this thread
// delivered.
template <bool MOD>
__device__ unsigned segment_walk(const WalkArgs& a, SegHead& head, int* sP, float* sX, int j, int k, int e,
                                 bool deliver, int now, int m_new, int tid) {
    __syncthreads();   // the block is done with the previous segment's lists
    const long long seg = static_cast<long long>(j) * a.nd + k;
    if (tid == 0) {
        SegHead h;
        h.s0 = static_cast<uint32_t>(a.seg_ptr[seg]);
        h.s1 = static_cast<uint32_t>(a.seg_ptr[seg + 1]);
        h.T = a.seg_last[seg];
        h.xT = a.seg_x[seg];
        const int4 rj = a.src_recent[j];
        h.nP = -2;
        if (h.T < e) {
            if (e - h.T > kMaxSpan) {
                h.nP = -1;
                set_err(a.err, ERR_SNAPSHOT);
            } else {
                const bool own = j >= a.src_lo && j < a.src_hi;
                h.nP = spikes_in(rj, own ? a.src_ring : nullptr, a.src_cnt, j - a.src_lo, a.ring_k, h.T, e, sP, kMaxPre);
                if (h.nP < 0) {
                    h.nP = -1;
                    set_err(a.err, ERR_HISTORY);
                }
            }
        }
        head = h;
    }
    __syncthreads();
    const SegHead h = head;
    const uint32_t len = h.s1 - h.s0;
    // the first round's synapses, independent of the segment's history
    uint32_t t_first = 0;
    float w_first = 0.0f;
    if (static_cast<uint32_t>(tid) < len) {
        t_first = __ldcs(a.tgt + h.s0 + tid);
        w_first = a.w[h.s0 + tid];
    }
    unsigned n = 0;
    if (h.nP >= 0) {
        Seg g;
        g.j = j;
        g.seg = seg;
        g.s0 = h.s0;
        g.s1 = h.s1;
        g.T = h.T;
        g.e = e;
        g.P.p = sP;
        g.P.n = h.nP;
        g.X = sX;
        build_table(a, g, sX, h.xT, m_new, tid);
        __syncthreads();
        if (tid == 0) finish_seg(a, g);
        n = walk_block<MOD>(a, g, deliver, now, tid, t_first, w_first);
    } else if (deliver) {
        // nothing to apply (or a history error, flagged): deliver only
        if (static_cast<uint32_t>(tid) < len) {
            atomicAdd(a.acc + t_first, MOD ? w_first * __ldg(a.mod + h.s0 + tid) : w_first);
            ++n;
        }
        for (uint32_t o = tid + kThreads; o < len; o += kThreads) {
            const uint32_t syn = h.s0 + o;
            const float wv = a.w[syn];
            atomicAdd(a.acc + __ldg(a.tgt + syn), MOD ? wv * __ldg(a.mod + syn) : wv);
            ++n;
        }
    }
    return n;
}

// Segments [g0, g0 + count) (count <= kThreads) through e: each thread
// looks at one and the block walks, one after another, those with updates
// to apply -- all of them (flush), or (sweep) those not walked for `stale`
// steps whose source has no spike still to arrive.
template <bool MOD>
__device__ void segment_group(const WalkArgs& a, SegHead& head, int* sP, float* sX, int* list, int* n_list,
                              long long g0, int count, int e, bool sweep, int now, int m_new, int tid) {
    __syncthreads();   // the previous group's list is read
    if (tid == 0) *n_list = 0;
    __syncthreads();
    if (tid < count) {
        const long long seg = g0 + tid;
        const int j = static_cast<int>(seg / a.nd);
        const int T = a.seg_last[seg];
        bool go = T < e && a.seg_ptr[seg + 1] > a.seg_ptr[seg];
        if (sweep) {
            const int newest = a.src_recent[j].x;
            go = go && newest < now - (a.dmin + a.nd - 1) && T < now - a.stale;
        }
        if (go) list[atomicAdd(n_list, 1)] = tid;
    }
    __syncthreads();
    const int n = *n_list;
    for (int q = 0; q < n; ++q) {
        const long long seg = g0 + list[q];
        segment_walk<MOD>(a, head, sP, sX, static_cast<int>(seg / a.nd), static_cast<int>(seg % a.nd), e, false, now,
                          m_new, tid);
    }
}

constexpr int kGroup = 8;   // segments a sweep unit looks at

template <bool MOD>
__global__ void __launch_bounds__(kThreads, kMinBlocks) walk_kernel(const __grid_constant__ WalkArgs a, int mode,
                                                                  long long step_off, const long long* step_base) {
    using Scan = cub::BlockScan<long long, kThreads>;
    __shared__ typename Scan::TempStorage scan_tmp;
    __shared__ long long start[257];
    __shared__ int slot[256];
    __shared__ int sP[kMaxPre];
    __shared__ float sX[kMaxSpan];
    __shared__ SegHead head;
    __shared__ int list[kThreads];
    __shared__ int n_list;

    const int tid = threadIdx.x;
    const long long step = step_off + (step_base ? *step_base : 0);
    const int now = static_cast<int>(step);
    const int m_new = static_cast<int>(step / a.win);   // newest snapshot written
    const long long n_seg = static_cast<long long>(a.n_src) * a.nd;

    if (mode == WALK_FLUSH) {
        // every segment through step - 1
        for (long long g0 = static_cast<long long>(blockIdx.x) * kThreads; g0 < n_seg;
             g0 += static_cast<long long>(gridDim.x) * kThreads) {
            const int count = n_seg - g0 < kThreads ? static_cast<int>(n_seg - g0) : kThreads;
            segment_group<MOD>(a, head, sP, sX, list, &n_list, g0, count, now - 1, false, now, m_new, tid);
        }
        return;
    }

    // Arrivals: spikes of step - (dmin + k) through the delay-k segments,
    // one unit each.
    long long units = 0;
    if (tid < a.nd) {
        const long long src_step = step - (a.dmin + tid);
        slot[tid] = src_step >= 0 ? static_cast<int>(src_step % a.hist_src.depth) : 0;
        if (src_step >= 0) units = a.hist_src.count[slot[tid]];
    }
    long long excl, n_arr;
    Scan(scan_tmp).ExclusiveSum(units, excl, n_arr);
    if (tid < a.nd) start[tid] = excl;
    if (tid == 0) start[a.nd] = n_arr;
    __syncthreads();

    // Sweep: the segments of rows [r0, r0 + rows), kGroup per unit.
    const long long r0 = (step % a.sweep_period) * a.sweep_rows;
    const long long left = a.n_src - r0;
    const long long rows = left <= 0 ? 0 : (a.sweep_rows < left ? a.sweep_rows : left);
    const long long sweep_segs = rows * a.nd;
    const long long n_units = n_arr + (sweep_segs + kGroup - 1) / kGroup;
    const int win_end = static_cast<int>((step / a.win) * a.win) - 1;   // spikes of all ranks known through here

    unsigned long long my_events = 0;
    for (long long u = blockIdx.x; u < n_units; u += gridDim.x) {
        if (u < n_arr) {
            int lo = 0, hi = a.nd - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (start[mid] <= u) lo = mid; else hi = mid - 1;
            }
            const int k = lo;
            const int spike = static_cast<int>(u - start[k]);
            const int j = a.hist_src.ids[static_cast<long long>(slot[k]) * a.hist_src.cap + spike];
            my_events += segment_walk<MOD>(a, head, sP, sX, j, k, now - 1, true, now, m_new, tid);
        } else {
            const long long q0 = (u - n_arr) * kGroup;
            const int count = sweep_segs - q0 < kGroup ? static_cast<int>(sweep_segs - q0) : kGroup;
            segment_group<MOD>(a, head, sP, sX, list, &n_list, r0 * a.nd + q0, count, win_end, true, now, m_new, tid);
        }
    }
    // thread sums -> one atomic per warp
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) my_events += __shfl_down_sync(0xffffffffu, my_events, o);
    if (a.events && (tid & 31) == 0 && my_events) atomicAdd(a.events, my_events);
}

}  // namespace

nrn_status_t walk_launch(const WalkArgs& a, int mode, long long step_off, const long long* step_base,
                         cudaStream_t s) {
    NRN_CHECK_ARG(a.nd >= 1 && a.nd <= 256, "plastic projection: at most 256 delay values");
    NRN_CHECK_ARG(a.win >= 1 && a.sweep_period >= 1, "plastic projection: bad window or sweep period");
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
