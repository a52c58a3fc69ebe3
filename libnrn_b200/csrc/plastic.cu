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
// Work: each block is a two-stage pipeline over its units.  Warp 0 (the
// producer) prepares the next segment to walk -- state, source spike
// steps, source trace table, new segment state, L2 prefetch of the
// synapses -- while warps 1.. (the consumers) walk the current one, the
// two buffers swapping at one block barrier per segment.  Units: one per
// (arriving spike, segment); sweep and flush units are groups of segments
// that the producer looks at one lane each.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>

#include <cub/block/block_scan.cuh>

#include "common.cuh"
#include "internal.h"

namespace nrn {
namespace {

constexpr int kThreads = 256;
constexpr int kMinBlocks = 1024 / kThreads;   // 64 registers a thread
constexpr int kPairsPer = (256 + kThreads - 1) / kThreads;   // delay values per thread in the prologue
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
__device__ __noinline__ float walk_syn_long(const WalkArgs& a, int j, int T, int e, const int* P, int nP,
                                            const float* X, uint32_t i, int4 r, float w, float mod, int now,
                                            float xp0) {
    Seg g;
    g.j = j;
    g.T = T;
    g.e = e;
    g.P.p = P;
    g.P.n = nP;
    g.X = X;
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
    return walk_syn_long<MOD>(a, g.j, g.T, g.e, g.P.p, g.P.n, g.X, i, r, w, mod, now, xp0);
}

// The source trace over (T, e] into a shared table by one warp, window by
// window (one window per lane) from the snapshot at the window's start --
// or, for the first, from x_pre(T) -- with the same operations as the
// per-step update.
__device__ __forceinline__ void build_table(const WalkArgs& a, const Seg& g, float* sX, float xT, int m_new,
                                            int lane) {
    const int W = a.win, e = g.e;
    const int m0 = (g.T + 1) / W + 1;   // window ends b = m*W - 1 in (T, e): m = m0, m0+1, ...
    const int n_pieces = 1 + (m0 * W - 1 < e ? (e - (m0 * W - 1) + W - 1) / W : 0);
    // a lane's pieces kBatch at a time, their snapshot loads issued together
    // (short windows make many pieces: one per step for a one-step window)
    constexpr int kBatch = 4;
    for (int pc0 = lane; pc0 < n_pieces; pc0 += 32 * kBatch) {
        float xs[kBatch];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
            const int pc = pc0 + 32 * b;
            xs[b] = xT;
            if (pc > 0 && pc < n_pieces) {
                const int m = m0 + pc - 1;
                if (m_new - m >= a.pre_depth) set_err(a.err, ERR_SNAPSHOT);
                xs[b] = __ldg(a.pre_snap + static_cast<long long>(m & (a.pre_depth - 1)) * a.n_src + g.j);
            }
        }
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
            const int pc = pc0 + 32 * b;
            if (pc >= n_pieces) break;
            const int start = pc == 0 ? g.T : (m0 + pc - 1) * W - 1;
            float x = xs[b];
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
}

constexpr int kConsumers = kThreads - 32;   // threads that walk synapses (warps 1..)
constexpr int kGroup = 4;                    // segments a sweep or flush unit looks at

__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// Walks the segment's synapses, consumer thread c taking offsets c, c +
// kConsumers, ...; with deliver, adds the updated weights into the target
// accumulators.
template <bool MOD>
__device__ __forceinline__ unsigned walk_block(const WalkArgs& a, const Seg& g, bool deliver, int now, int c) {
    // the target trace at the first source spike is loaded with the target's spike steps
    const bool has_pre = g.P.n > 0;
    const int t0 = has_pre ? g.P[0] : 0;
    const float* ring0 = a.post_ring + static_cast<long long>(t0 & (a.post_depth - 1)) * a.n_tgt;
    // the next round's target and weight (the HBM stream) are loaded a round
    // ahead; the target's spike steps and trace (L2) within the round
    unsigned n = 0;
    const uint32_t len = g.s1 - g.s0;   // a projection holds < 2^32 synapses
    uint32_t t_next = 0;
    float w_next = 0.0f;
    if (static_cast<uint32_t>(c) < len) {
        t_next = __ldcs(a.tgt + g.s0 + c);
        w_next = a.w[g.s0 + c];
    }
#pragma unroll 1
    for (uint32_t o = c; o < len; o += kConsumers) {
        const uint32_t syn = g.s0 + o;
        const uint32_t t = t_next;
        const float w = w_next;
        const int4 r = a.tgt_recent[t];
        const float xp0 = has_pre ? ring0[t] : 0.0f;
        const float md = MOD ? __ldcs(a.mod + syn) : 1.0f;
        if (o + kConsumers < len) {
            t_next = __ldcs(a.tgt + syn + kConsumers);
            w_next = a.w[syn + kConsumers];
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

// Delivery without updates (the segment is up to date, or its history was
// flagged as an error).
template <bool MOD>
__device__ __forceinline__ unsigned deliver_only(const WalkArgs& a, uint32_t s0, uint32_t s1, int c) {
    unsigned n = 0;
    for (uint32_t o = c; o < s1 - s0; o += kConsumers) {
        const uint32_t syn = s0 + o;
        const float wv = a.w[syn];
        atomicAdd(a.acc + __ldg(a.tgt + syn), MOD ? wv * __ldg(a.mod + syn) : wv);
        ++n;
    }
    return n;
}

// New segment state after a walk through g.e.
__device__ __forceinline__ void finish_seg(const WalkArgs& a, const Seg& g) {
    a.seg_x[g.seg] = g.X[g.e - g.T - 1];
    a.seg_last[g.seg] = g.e;
}

enum { ITEM_DONE = 0, ITEM_WALK = 1, ITEM_DELIVER = 2 };

// One segment walk, prepared by the producer warp for the consumers.
struct Item {
    int kind;
    int j, T, e, nP, deliver;
    uint32_t s0, s1;
};

// What the producer warp needs to step through the block's units.
struct Producer {
    unsigned int* ctr;    // the launch's unit counter (units are taken dynamically)
    long long u;          // unused (kept for the layout of the shared state)
    long long n_units, n_arr;
    long long base, g_end;   // group units cover segments [base, g_end), kGroup each
    unsigned pending;     // segments g0 + bit of the current group still to look at
    long long g0;
    int e_group;          // groups walk through this step
};

// Segment (j, k) through e, by the producer warp: state and source spike
// steps (lane 0, one round trip), the source trace table (all lanes, one
// round trip for the snapshots), the segment's new state, and an L2
// prefetch of its synapses for the consumers.  Returns false when there is
// nothing to walk or deliver (a sweep or flush segment already up to date).
__device__ bool prepare(const WalkArgs& a, Item& it, int* sP, float* sX, int j, int k, int e, bool deliver, int now,
                        int m_new, int lane) {
    const long long seg = static_cast<long long>(j) * a.nd + k;
    Item h;
    h.kind = ITEM_DONE;
    h.j = j;
    h.e = e;
    h.deliver = deliver;
    int nP = -2;
    float xT = 0.0f;
    if (lane == 0) {
        h.s0 = static_cast<uint32_t>(a.seg_ptr[seg]);
        h.s1 = static_cast<uint32_t>(a.seg_ptr[seg + 1]);
        h.T = a.seg_last[seg];
        xT = a.seg_x[seg];
        const int4 rj = a.src_recent[j];
        if (h.T < e) {
            if (e - h.T > kMaxSpan) {
                nP = -1;
                set_err(a.err, ERR_SNAPSHOT);
            } else {
                const bool own = j >= a.src_lo && j < a.src_hi;
                nP = spikes_in(rj, own ? a.src_ring : nullptr, a.src_cnt, j - a.src_lo, a.ring_k, h.T, e, sP, kMaxPre);
                if (nP < 0) {
                    nP = -1;
                    set_err(a.err, ERR_HISTORY);
                }
            }
        }
    }
    nP = __shfl_sync(0xffffffffu, nP, 0);
    h.s0 = __shfl_sync(0xffffffffu, h.s0, 0);
    h.s1 = __shfl_sync(0xffffffffu, h.s1, 0);
    h.T = __shfl_sync(0xffffffffu, h.T, 0);
    xT = __shfl_sync(0xffffffffu, xT, 0);
    h.nP = nP;
    __syncwarp();   // sP written by lane 0
    if (nP >= 0) {
        h.kind = ITEM_WALK;
        if (nP > 0 && now - sP[0] >= a.post_depth) set_err(a.err, ERR_SNAPSHOT);
        Seg g;
        g.j = j;
        g.seg = seg;
        g.T = h.T;
        g.e = e;
        g.P.p = sP;
        g.P.n = nP;
        g.X = sX;
        build_table(a, g, sX, xT, m_new, lane);
        __syncwarp();
        if (lane == 0) finish_seg(a, g);
    } else if (deliver) {
        h.kind = ITEM_DELIVER;
    } else {
        return false;
    }
    // the consumers' first rounds come from L2
    for (uint32_t o = h.s0 + 32u * lane; o < h.s1; o += 32u * 32u) {
        prefetch_l2(a.tgt + o);
        prefetch_l2(a.w + o);
        if (a.mod) prefetch_l2(a.mod + o);
    }
    if (lane == 0) it = h;
    return true;
}

// The producer's next item into `it` (kind ITEM_DONE when the block's
// units are exhausted).  Arrival units give one item each; sweep and flush
// units are groups of kGroup segments, looked at one lane each, whose
// segments to walk become items one after another.  The producer's state
// lives in shared memory (only warp 0 reads it), so the consumers' loop
// does not carry it in registers.
__device__ void produce(const WalkArgs& a, Producer& shared_pr, Item& it, int* sP, float* sX, const long long* start,
                        const int* slot, bool sweep, int now, int m_new, int lane) {
    Producer pr = shared_pr;
    for (;;) {
        bool got = false;
        while (pr.pending && !got) {
            const int b = __ffs(pr.pending) - 1;
            pr.pending &= pr.pending - 1;
            const long long seg = pr.g0 + b;
            got = prepare(a, it, sP, sX, static_cast<int>(seg / a.nd), static_cast<int>(seg % a.nd), pr.e_group, false,
                          now, m_new, lane);
        }
        if (got) break;
        // The next unit of the launch, taken from its counter: blocks that
        // finish early take more, so uneven units (sweep groups walk 0 to
        // kGroup segments) do not leave a tail.  Sweep and flush groups come
        // first, arrivals (all about the same size) after them.
        unsigned int k = 0;
        if (lane == 0) k = atomicAdd(pr.ctr, 1u);
        k = __shfl_sync(0xffffffffu, k, 0);
        if (static_cast<long long>(k) >= pr.n_units) {
            if (lane == 0) it.kind = ITEM_DONE;
            break;
        }
        const long long n_grp = pr.n_units - pr.n_arr;
        const long long u = static_cast<long long>(k) < n_grp ? pr.n_arr + k : static_cast<long long>(k) - n_grp;
        if (u < pr.n_arr) {
            int lo = 0, hi = a.nd - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (start[mid] <= u) lo = mid; else hi = mid - 1;
            }
            const int spike = static_cast<int>(u - start[lo]);
            const int j = a.hist_src.ids[static_cast<long long>(slot[lo]) * a.hist_src.cap + spike];
            // an item, except for an up-to-date segment when delivery is left
            // to the deterministic delivery
            if (prepare(a, it, sP, sX, j, lo, now - 1, a.no_deliver == 0, now, m_new, lane)) break;
            continue;
        }
        // a group of segments: each lane looks at one
        pr.g0 = pr.base + (u - pr.n_arr) * kGroup;
        const long long seg = pr.g0 + lane;
        bool go = false;
        if (lane < kGroup && seg < pr.g_end) {
            const int j = static_cast<int>(seg / a.nd);
            const int T = a.seg_last[seg];
            go = T < pr.e_group && a.seg_ptr[seg + 1] > a.seg_ptr[seg];
            if (sweep) {
                const int newest = a.src_recent[j].x;
                go = go && newest < now - (a.dmin + a.nd - 1) && T < now - a.stale;
            }
        }
        pr.pending = __ballot_sync(0xffffffffu, go);
    }
    __syncwarp();
    if (lane == 0) {   // the fields that change (the consumers read the others)
        shared_pr.u = pr.u;
        shared_pr.pending = pr.pending;
        shared_pr.g0 = pr.g0;
    }
    __syncwarp();
}

template <bool MOD>
__global__ void __launch_bounds__(kThreads, kMinBlocks) walk_kernel(const __grid_constant__ WalkArgs a, int mode,
                                                                  long long step_off, const long long* step_base) {
    using Scan = cub::BlockScan<long long, kThreads>;
    __shared__ typename Scan::TempStorage scan_tmp;
    __shared__ long long start[257];
    __shared__ int slot[256];
    __shared__ int sP[2][kMaxPre];
    __shared__ float sX[2][kMaxSpan];
    __shared__ Item items[2];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long step = step_off + (step_base ? *step_base : 0);
    const int now = static_cast<int>(step);
    const int m_new = static_cast<int>(step / a.win);   // newest snapshot written
    const long long n_seg = static_cast<long long>(a.n_src) * a.nd;

    __shared__ Producer pr;
    bool sweep = false;
    if (mode == WALK_FLUSH) {
        // every segment through step - 1, kGroup per unit
        if (tid == 0) {
            pr.n_arr = 0;
            pr.n_units = (n_seg + kGroup - 1) / kGroup;
            pr.base = 0;
            pr.g_end = n_seg;
            pr.e_group = now - 1;
        }
    } else {
        // Arrivals: spikes of step - (dmin + k) through the delay-k
        // segments, one unit each; then the sweep: the segments of rows
        // [r0, r0 + rows), kGroup per unit.
        long long units[kPairsPer];
#pragma unroll
        for (int r = 0; r < kPairsPer; ++r) {
            const int k = tid * kPairsPer + r;   // the scan's blocked arrangement
            units[r] = 0;
            if (k < a.nd) {
                const long long src_step = step - (a.dmin + k);
                slot[k] = src_step >= 0 ? static_cast<int>(src_step % a.hist_src.depth) : 0;
                if (src_step >= 0) units[r] = a.hist_src.count[slot[k]];
            }
        }
        long long excl[kPairsPer], n_arr;
        Scan(scan_tmp).ExclusiveSum(units, excl, n_arr);
#pragma unroll
        for (int r = 0; r < kPairsPer; ++r)
            if (tid * kPairsPer + r < a.nd) start[tid * kPairsPer + r] = excl[r];
        if (tid == 0) {
            start[a.nd] = n_arr;
            const long long r0 = (step % a.sweep_period) * a.sweep_rows;
            const long long left = a.n_src - r0;
            const long long rows = left <= 0 ? 0 : (a.sweep_rows < left ? a.sweep_rows : left);
            pr.n_arr = n_arr;
            pr.n_units = n_arr + (rows * a.nd + kGroup - 1) / kGroup;
            pr.base = r0 * a.nd;
            pr.g_end = (r0 + rows) * a.nd;
            pr.e_group = static_cast<int>((step / a.win) * a.win) - 1;   // spikes of all ranks known through here
        }
        sweep = true;
    }
    if (tid == 0) {
        // unit counters: [0], [1] by step parity (each step's launch clears
        // the other's for the next step), [2] for flushes (cleared by the host)
        const int slot = mode == WALK_FLUSH ? 2 : static_cast<int>(step & 1);
        pr.ctr = a.work_ctr + slot;
        if (blockIdx.x == 0 && mode != WALK_FLUSH) a.work_ctr[(step + 1) & 1] = 0u;
        pr.u = 0;
        pr.pending = 0;
        pr.g0 = 0;
    }
    __syncthreads();

    if (warp == 0) {
        produce(a, pr, items[0], sP[0], sX[0], start, slot, sweep, now, m_new, lane);
    } else if (sweep) {
        // Meanwhile the consumers bring into L2 what the producer will read
        // for this block's later arrival units: segment bounds and state,
        // and source spike steps.
        const long long u = blockIdx.x + static_cast<long long>(tid - 32 + 1) * gridDim.x;
        if (u < pr.n_arr) {
            int lo = 0, hi = a.nd - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (start[mid] <= u) lo = mid; else hi = mid - 1;
            }
            const int j = a.hist_src.ids[static_cast<long long>(slot[lo]) * a.hist_src.cap + (u - start[lo])];
            const long long seg = static_cast<long long>(j) * a.nd + lo;
            prefetch_l2(a.seg_ptr + seg);
            prefetch_l2(a.seg_last + seg);
            prefetch_l2(a.seg_x + seg);
            prefetch_l2(a.src_recent + j);
        }
    }
    __syncthreads();
    unsigned long long my_events = 0;
    for (int q = 0;; q ^= 1) {
        const Item cur = items[q];
        if (cur.kind == ITEM_DONE) break;
        if (warp == 0) {
            produce(a, pr, items[q ^ 1], sP[q ^ 1], sX[q ^ 1], start, slot, sweep, now, m_new, lane);
        } else if (cur.kind == ITEM_WALK) {
            Seg g;
            g.j = cur.j;
            g.seg = 0;
            g.s0 = cur.s0;
            g.s1 = cur.s1;
            g.T = cur.T;
            g.e = cur.e;
            g.P.p = sP[q];
            g.P.n = cur.nP;
            g.X = sX[q];
            my_events += walk_block<MOD>(a, g, cur.deliver != 0, now, tid - 32);
        } else {
            my_events += deliver_only<MOD>(a, cur.s0, cur.s1, tid - 32);
        }
        __syncthreads();
    }
    // thread sums -> one atomic per warp
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) my_events += __shfl_down_sync(0xffffffffu, my_events, o);
    if (a.events && lane == 0 && my_events) atomicAdd(a.events, my_events);
}

}  // namespace

nrn_status_t walk_launch(const WalkArgs& a, int mode, long long step_off, const long long* step_base,
                         cudaStream_t s) {
    NRN_CHECK_ARG(a.nd >= 1 && a.nd <= 256, "plastic projection: at most 256 delay values");
    NRN_CHECK_ARG(a.win >= 1 && a.sweep_period >= 1, "plastic projection: bad window or sweep period");
    NRN_CHECK_ARG(a.work_ctr != nullptr, "plastic projection: no unit counters");
    if (mode == WALK_FLUSH) NRN_CUDA_TRY(cudaMemsetAsync(a.work_ctr + 2, 0, sizeof(unsigned int), s));
    NRN_CHECK_ARG(a.pre_depth > 0 && (a.pre_depth & (a.pre_depth - 1)) == 0 && a.post_depth > 0 &&
                      (a.post_depth & (a.post_depth - 1)) == 0,
                  "plastic projection: trace ring depths must be powers of two");
    auto launch = [&](auto kern) -> nrn_status_t {
        int per_sm = 0;
        NRN_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, 0));
        kern<<<std::max(1, per_sm) * sm_count_current(), kThreads, 0, s>>>(a, mode, step_off, step_base);
        NRN_CUDA_TRY(cudaGetLastError());
        return NRN_OK;
    };
    return a.mod ? launch(walk_kernel<true>) : launch(walk_kernel<false>);
}

}  // namespace nrn
