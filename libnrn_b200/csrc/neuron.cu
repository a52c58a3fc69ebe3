// neuron.cu -- fused per-population neuron update (LIF, AdEx, Izhikevich).
//
// One thread per neuron: read the input (current and, for AdEx, conductance
// input), add the external drive, integrate one step, detect the spike,
// write state, zero the consumed input, and append spiking ids with one
// warp-ballot compaction (one atomic per warp that has a spike).
//
// Each model's arithmetic restates the reference's CPU path operation by
// operation (src/neuron/lif.cpp:80-97, src/neuron/adex.cpp:97-124,
// src/neuron/izhikevich.cpp:76-98): this file is compiled with -fmad=false,
// so every multiply and add rounds on its own as the torch ops do, and
// scalars the reference passes as doubles are rounded to float on the host.
//
// Memory per neuron and step (uniform parameters): LIF 28 B, Izhikevich
// 28 B (+20 B per-neuron a,b,c,d,v_peak), AdEx with conductances 64 B.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "rng.cuh"

namespace nrn {
namespace {

struct PopArgs {
    int n;
    int gid_offset;
    float dtf;                 // (float)dt
    float half, dtm;           // Izhikevich: (float)(0.5*dt_ms), (float)dt_ms
    float dec_e, dec_i;        // conductance decay per step
    float e_exc, e_inh;
    float* v;
    float* aux;
    float* ref;
    float* spike;
    float* i_syn;
    float* g_exc;
    float* g_inh;
    float* gin_exc;
    float* gin_inh;
    const float* param[NRN_MAX_PARAMS];
    float uniform[NRN_MAX_PARAMS];
    int drive_kind;
    float d0, d1, d_exp;       // drive parameters, expf(-lambda)
    // Poisson CDF F_0..F_{n_cdf-1} of the drive, built on the host with the
    // sampler's own float operations (p_k = p_{k-1}*lambda/k, F_k = F_{k-1}+p_k)
    float cdf[32];
    int n_cdf;
    const float* drive_values;   // this step's drive drawn ahead, or null
    nrn_spike_stat_t* spike_stats;   // per-neuron spike statistics, or null
    uint64_t seed;
    int64_t step;
    const int64_t* step_base;
    int* spike_ids;
    int* spike_count;
    int hist_depth;
    int hist_cap;
    int* raster_step;
    int* raster_gid;
    unsigned long long* raster_count;
    long long raster_cap;
    int n_traces;
    int trace_slow_ratio;
    float* trace[NRN_MAX_TRACES];
    float trace_decay[NRN_MAX_TRACES];
    float* trace_ring[NRN_MAX_TRACES];
    int trace_ring_depth;
    int4* post_recent;
    int* post_ring;
    int* post_cnt;
    int post_ring_k;
    int id_offset;
    int win;
    uint32_t* win_mask;
    int* send_hdr;
    int* send_ids;
    int send_cap;
    int* err;
    int n_chan;                // synapse channels
    int chan_kind[4];
    float chan_dec_rise[4], chan_dec_decay[4], chan_e_rev[4];
    float* chan_in[4];
    float* chan_s[4];
    float* chan_r[4];
};

// This step's synapse channel currents added to I (nrn_syn_desc_t), the
// channel input consumed; v is the potential before the update.
__device__ __forceinline__ float apply_channels(const PopArgs& a, int i, float I, float v) {
    for (int c = 0; c < a.n_chan; ++c) {
        const float in = a.chan_in[c][i];
        a.chan_in[c][i] = 0.0f;
        const float sd = a.chan_s[c][i] * a.chan_dec_decay[c] + in;
        a.chan_s[c][i] = sd;
        if (a.chan_kind[c] == NRN_SYN_EXP) {
            I = I + sd;
            continue;
        }
        const float sr = a.chan_r[c][i] * a.chan_dec_rise[c] + in;
        a.chan_r[c][i] = sr;
        const float g = sd - sr;
        I = a.chan_kind[c] == NRN_SYN_DEXP ? I + g : I + g * (a.chan_e_rev[c] - v);
    }
    return I;
}

template <bool HET>
__device__ __forceinline__ float par(const PopArgs& a, int k, int i) {
    if (HET) {
        const float* p = a.param[k];
        return p ? __ldg(p + i) : a.uniform[k];
    }
    return a.uniform[k];
}

// Poisson count of the drive from its uniform: the first k with u <= F_k,
// from the table (the same values the loop of poisson_inv adds up); past
// the table, the loop itself.
__device__ __forceinline__ float poisson_drive(const PopArgs& a, uint32_t word) {
    const float u = u01(word);
    int k = 0;
    while (k < a.n_cdf && u > a.cdf[k]) ++k;
    if (k == a.n_cdf) k = poisson_inv(u, a.d0, a.d_exp);
    return a.d1 * static_cast<float>(k);
}

__device__ __forceinline__ uint32_t word_at(const U4& w, uint32_t q) {
    return q == 0 ? w.x : q == 1 ? w.y : q == 2 ? w.z : w.w;
}

// The drive of neuron gid at step.  Poisson kinds: word gid % 4 of the
// Philox block (gid / 4, step) -- four consecutive neurons share a block;
// Gaussian: words 0 and 1 of the block (gid, step).
__device__ __forceinline__ float drive_value(const PopArgs& a, uint32_t gid, uint32_t step) {
    if (a.drive_kind == NRN_DRIVE_GAUSS_CURRENT) {
        const U4 w = philox4x32_10(U4{gid, step, 0u, kStreamDrive}, a.seed);
        float z = normal_bm(u01(w.x), u01(w.y));
        return a.d0 + a.d1 * z;
    }
    const U4 w = philox4x32_10(U4{gid >> 2, step, 0u, kStreamDrive}, a.seed);
    return poisson_drive(a, word_at(w, gid & 3u));
}

// The drive of neurons gid0 .. gid0+3 (one Philox block when gid0 is a
// multiple of 4 and the drive is Poisson).
__device__ __forceinline__ float4 drive_value4(const PopArgs& a, uint32_t gid0, uint32_t step) {
    if (a.drive_kind != NRN_DRIVE_GAUSS_CURRENT && (gid0 & 3u) == 0) {
        const U4 w = philox4x32_10(U4{gid0 >> 2, step, 0u, kStreamDrive}, a.seed);
        return make_float4(poisson_drive(a, w.x), poisson_drive(a, w.y), poisson_drive(a, w.z), poisson_drive(a, w.w));
    }
    return make_float4(drive_value(a, gid0, step), drive_value(a, gid0 + 1, step), drive_value(a, gid0 + 2, step),
                       drive_value(a, gid0 + 3, step));
}

// A spike of neuron i at step t into its statistics: count, and the
// interval since its previous spike (exact integer sums).
__device__ __forceinline__ void record_spike_stat(nrn_spike_stat_t* s, int i, int t) {
    nrn_spike_stat_t r = s[i];
    if (r.last > 0) {
        const long long isi = static_cast<long long>(t) + 1 - r.last;
        r.isi_sum += isi;
        r.isi_sum2 += isi * isi;
    }
    r.last = t + 1;
    r.count += 1;
    s[i] = r;
}

// The LIF update of one neuron (src/neuron/lif.cpp:80-97), each operation
// rounded to fp32 in the reference's order; returns whether it spiked.
__device__ __forceinline__ bool lif_math(float v, float ref, float I, float dtf, float v_rest, float v_th,
                                         float v_reset, float tau_m, float tau_ref, float c_m, float i_bg, float& vn_out,
                                         float& r_out) {
    const bool active = ref <= 0.0f;
    float r = ref > 0.0f ? ref - dtf : ref;
    float lk = (-(v - v_rest)) / tau_m;
    float in = (I + i_bg) / c_m;
    float dv = dtf * (lk + in);
    float vn = active ? v + dv : v;
    const bool spiked = (vn >= v_th) && active;
    if (spiked) { vn = v_reset; r = tau_ref; }
    vn_out = vn;
    r_out = r;
    return spiked;
}

// One neuron of one population: every thread of a warp belongs to the same
// population (the compaction below is warp-wide).
template <int MODEL, bool HET, bool COND>
__device__ __forceinline__ void pop_body(const PopArgs& a, const int i) {
    const bool valid = i < a.n;
    int spiked = 0;
    long long step = a.step;
    if (a.step_base) step += *a.step_base;
    if (valid) {
        float I = a.i_syn ? a.i_syn[i] : 0.0f;
        float in_e = 0.0f, in_i = 0.0f;
        if (COND) {
            in_e = a.gin_exc[i];
            in_i = a.gin_inh[i];
        }
        if (a.drive_kind != NRN_DRIVE_NONE) {
            const float x = a.drive_values ? a.drive_values[i]
                                           : drive_value(a, static_cast<uint32_t>(a.gid_offset + i),
                                                         static_cast<uint32_t>(step));
            if (a.drive_kind == NRN_DRIVE_POISSON_GEXC) in_e = in_e + x;
            else I = I + x;
        }
        if (a.n_chan > 0) I = apply_channels(a, i, I, a.v[i]);
        if (MODEL == NRN_MODEL_LIF) {
            float v = a.v[i], ref = a.ref[i];
            const float v_rest = par<HET>(a, 0, i), v_th = par<HET>(a, 1, i);
            const float v_reset = par<HET>(a, 2, i), tau_m = par<HET>(a, 3, i);
            const float tau_ref = par<HET>(a, 4, i), c_m = par<HET>(a, 5, i);
            const float i_bg = par<HET>(a, 6, i);
            float vn, r;
            spiked = lif_math(v, ref, I, a.dtf, v_rest, v_th, v_reset, tau_m, tau_ref, c_m, i_bg, vn, r);
            a.v[i] = vn;
            a.ref[i] = r;
        } else if (MODEL == NRN_MODEL_ADEX) {
            float v = a.v[i], w = a.aux[i], ref = a.ref[i];
            if (COND) {
                float ge = a.g_exc[i] * a.dec_e + in_e;
                float gi = a.g_inh[i] * a.dec_i + in_i;
                a.g_exc[i] = ge;
                a.g_inh[i] = gi;
                I = I + ge * (a.e_exc - v);
                I = I + gi * (a.e_inh - v);
            }
            const float v_rest = par<HET>(a, 0, i), v_th = par<HET>(a, 1, i);
            const float v_reset = par<HET>(a, 2, i), v_peak = par<HET>(a, 3, i);
            const float tau_w = par<HET>(a, 5, i), tau_ref = par<HET>(a, 6, i);
            const float c_m = par<HET>(a, 7, i), g_l = par<HET>(a, 8, i);
            const float pa = par<HET>(a, 9, i), pb = par<HET>(a, 10, i);
            const float delta_t = par<HET>(a, 11, i), i_bg = par<HET>(a, 12, i);
            const bool active = ref <= 0.0f;
            float r = ref > 0.0f ? ref - a.dtf : ref;
            // exp in double, rounded once to float: the correctly rounded
            // float exp in all but rare cases, as the reference's CPU exp.
            const float ex = static_cast<float>(exp(static_cast<double>((v - v_th) / delta_t)));
            float I_exp = (g_l * delta_t) * ex;
            float acc = (-g_l) * (v - v_rest);
            acc = acc + I_exp;
            acc = acc - w;
            acc = acc + I;
            acc = acc + i_bg;
            float dv = (a.dtf * acc) / c_m;
            float vn = active ? v + dv : v;
            float dw = (a.dtf * ((pa * (vn - v_rest)) - w)) / tau_w;
            float wn = w + dw;
            spiked = (vn >= v_peak) && active;
            if (spiked) { vn = v_reset; wn = wn + pb; r = tau_ref; }
            a.v[i] = vn;
            a.aux[i] = wn;
            a.ref[i] = r;
        } else {
            float v = a.v[i], u = a.aux[i];
            const float pa = par<HET>(a, 0, i), pb = par<HET>(a, 1, i);
            const float pc = par<HET>(a, 2, i), pd = par<HET>(a, 3, i);
            const float v_peak = par<HET>(a, 4, i);
            float dv1 = ((((0.04f * v) * v) + (5.0f * v)) + 140.0f - u) + I;
            v = v + a.half * dv1;
            float dv2 = ((((0.04f * v) * v) + (5.0f * v)) + 140.0f - u) + I;
            v = v + a.half * dv2;
            float du = (a.dtm * pa) * ((pb * v) - u);
            u = u + du;
            spiked = v >= v_peak;
            if (spiked) { v = pc; u = u + pd; }
            a.v[i] = v;
            a.aux[i] = u;
        }
        if (a.spike) a.spike[i] = spiked ? 1.0f : 0.0f;
        if (a.n_traces > 0 && (a.trace_slow_ratio <= 1 || step % a.trace_slow_ratio == 0)) {
            // pair-STDP traces (src/plasticity/stdp.cpp:118-128): decay, then + spike
            const float sp = spiked ? 1.0f : 0.0f;
            for (int k = 0; k < a.n_traces; ++k) {
                if (a.trace_ring[k] != nullptr) {
                    const long long mask = a.trace_ring_depth - 1;   // depth is a power of two
                    const float prev = a.trace_ring[k][((step - 1) & mask) * a.n + i];
                    a.trace_ring[k][(step & mask) * a.n + i] = prev * a.trace_decay[k] + sp;
                } else {
                    a.trace[k][i] = a.trace[k][i] * a.trace_decay[k] + sp;
                }
            }
        }
        if (spiked && a.post_recent != nullptr) {
            const int t = static_cast<int>(step);
            int4 r = a.post_recent[i];
            a.post_recent[i] = make_int4(t, r.x, r.y, r.z);
            const int c = a.post_cnt[i];
            a.post_ring[static_cast<long long>(i) * a.post_ring_k + (c % a.post_ring_k)] = t;
            a.post_cnt[i] = c + 1;
        }
        if (spiked && a.win_mask != nullptr) a.win_mask[i] |= 1u << static_cast<int>(step % a.win);
        if (spiked && a.spike_stats != nullptr) record_spike_stat(a.spike_stats, i, static_cast<int>(step));
        if (a.i_syn) a.i_syn[i] = 0.0f;
        if (COND) {
            a.gin_exc[i] = 0.0f;
            a.gin_inh[i] = 0.0f;
        }
    }
    // Warp-ballot compaction: ascending ids within a warp, one atomic per warp.
    if (a.spike_ids != nullptr || a.send_hdr != nullptr || a.raster_gid != nullptr) {
        const unsigned mask = __ballot_sync(0xffffffffu, spiked);
        if (mask) {
            const int lane = threadIdx.x & 31;
            const int leader = __ffs(mask) - 1;
            const int cnt = __popc(mask);
            const int rank = __popc(mask & ((1u << lane) - 1u));
            if (a.send_hdr) {
                // window send buffer: ids in step order (the steps of a window
                // run one after the other), the running total in send_hdr[win]
                const int u = static_cast<int>(step % a.win);
                int base = 0;
                if (lane == leader) {
                    base = atomicAdd(a.send_hdr + a.win, cnt);
                    atomicAdd(a.send_hdr + u, cnt);
                }
                base = __shfl_sync(0xffffffffu, base, leader);
                if (spiked) {
                    if (base + rank < a.send_cap) a.send_ids[base + rank] = a.id_offset + i;
                    else if (a.err) atomicCAS(a.err, 0, 4);
                }
            } else if (a.spike_ids) {
                int* ids = a.spike_ids;
                int* count = a.spike_count;
                if (a.hist_depth > 0) {
                    const int slot = static_cast<int>(step % a.hist_depth);
                    ids += static_cast<long long>(slot) * a.hist_cap;
                    count += slot;
                }
                int base = 0;
                if (lane == leader) base = atomicAdd(count, cnt);
                base = __shfl_sync(0xffffffffu, base, leader);
                if (spiked) ids[base + rank] = a.id_offset + i;
            }
            if (a.raster_gid) {
                unsigned long long rb = 0;
                if (lane == leader) rb = atomicAdd(a.raster_count, static_cast<unsigned long long>(cnt));
                rb = __shfl_sync(0xffffffffu, rb, leader);
                const unsigned long long pos = rb + rank;
                if (spiked && pos < static_cast<unsigned long long>(a.raster_cap)) {
                    a.raster_step[pos] = static_cast<int>(step);
                    a.raster_gid[pos] = a.gid_offset + i;
                }
            }
        }
    }
}

template <int MODEL, bool HET, bool COND>
__global__ void __launch_bounds__(256) pop_step_kernel(const __grid_constant__ PopArgs a) {
    pop_body<MODEL, HET, COND>(a, blockIdx.x * blockDim.x + threadIdx.x);
}

// Several populations of the same kind in one launch, block ranges
// [start[q], start[q+1]) for population q.
constexpr int kMaxGroup = 4;
struct PopGroup {
    PopArgs p[kMaxGroup];
    int start[kMaxGroup + 1];
    int n;
};

template <int MODEL, bool HET, bool COND>
__global__ void __launch_bounds__(256) pop_group_kernel(const __grid_constant__ PopGroup g) {
    int q = 0;
    while (q + 1 < g.n && static_cast<int>(blockIdx.x) >= g.start[q + 1]) ++q;
    pop_body<MODEL, HET, COND>(g.p[q], (static_cast<int>(blockIdx.x) - g.start[q]) * blockDim.x + threadIdx.x);
}

constexpr int kPopThreads = 256;

__device__ __forceinline__ float4 ld4(const float* p, int i) { return *reinterpret_cast<const float4*>(p + i); }
__device__ __forceinline__ void st4(float* p, int i, float4 x) { *reinterpret_cast<float4*>(p + i) = x; }
__device__ __forceinline__ float& at(float4& x, int k) { return k == 0 ? x.x : k == 1 ? x.y : k == 2 ? x.z : x.w; }

// LIF with uniform parameters, four neurons per group (float4 state, n a
// multiple of 4, arrays 16-byte aligned), G groups per thread, blockDim.x*4
// neurons apart (coalesced): the same arithmetic as pop_body (lif_math),
// with wider memory transactions and the loads of all G groups issued
// before any is used.
template <int G>
__global__ void __launch_bounds__(256) lif4_group_kernel(const __grid_constant__ PopGroup g) {
    int q = 0;
    while (q + 1 < g.n && static_cast<int>(blockIdx.x) >= g.start[q + 1]) ++q;
    const PopArgs& a = g.p[q];
    const int stride = 4 * static_cast<int>(blockDim.x);
    const int ib = 4 * ((static_cast<int>(blockIdx.x) - g.start[q]) * G * static_cast<int>(blockDim.x) +
                        static_cast<int>(threadIdx.x));
    const int lane = threadIdx.x & 31;
    long long step = a.step;
    if (a.step_base) step += *a.step_base;
    const bool traces_now = a.n_traces > 0 && (a.trace_slow_ratio <= 1 || step % a.trace_slow_ratio == 0);
    const long long ring_mask = a.trace_ring_depth - 1;
    float4 I[G], v[G], ref[G], x0[G];
#pragma unroll
    for (int j = 0; j < G; ++j) {
        const int i0 = ib + j * stride;
        if (i0 >= a.n) continue;
        I[j] = a.i_syn ? ld4(a.i_syn, i0) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.drive_kind != NRN_DRIVE_NONE) {
            float4 x;
            if (a.drive_values) x = ld4(a.drive_values, i0);
            else x = drive_value4(a, static_cast<uint32_t>(a.gid_offset + i0), static_cast<uint32_t>(step));
            I[j].x = I[j].x + x.x; I[j].y = I[j].y + x.y; I[j].z = I[j].z + x.z; I[j].w = I[j].w + x.w;
        }
        v[j] = ld4(a.v, i0);
        ref[j] = ld4(a.ref, i0);
        // the first trace is loaded with the state (the stores below could
        // alias it, so it would otherwise wait for them)
        x0[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (traces_now)
            x0[j] = a.trace_ring[0] != nullptr ? ld4(a.trace_ring[0] + ((step - 1) & ring_mask) * a.n, i0)
                                               : ld4(a.trace[0], i0);
    }
    int sp[4 * G];
#pragma unroll
    for (int k = 0; k < 4 * G; ++k) sp[k] = 0;
    const float* u = a.uniform;
#pragma unroll
    for (int j = 0; j < G; ++j) {
        const int i0 = ib + j * stride;
        if (i0 >= a.n) continue;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float vn, r;
            sp[4 * j + k] = lif_math(at(v[j], k), at(ref[j], k), at(I[j], k), a.dtf, u[0], u[1], u[2], u[3], u[4],
                                     u[5], u[6], vn, r);
            at(v[j], k) = vn;
            at(ref[j], k) = r;
        }
        st4(a.v, i0, v[j]);
        st4(a.ref, i0, ref[j]);
        const float4 s4 = make_float4(sp[4 * j] ? 1.f : 0.f, sp[4 * j + 1] ? 1.f : 0.f, sp[4 * j + 2] ? 1.f : 0.f,
                                      sp[4 * j + 3] ? 1.f : 0.f);
        if (a.spike) st4(a.spike, i0, s4);
        if (traces_now) {
            for (int k = 0; k < a.n_traces; ++k) {
                const float d = a.trace_decay[k];
                float4 x;
                float* dst;
                if (a.trace_ring[k] != nullptr) {
                    x = k == 0 ? x0[j] : ld4(a.trace_ring[k] + ((step - 1) & ring_mask) * a.n, i0);
                    dst = a.trace_ring[k] + (step & ring_mask) * a.n;
                } else {
                    x = k == 0 ? x0[j] : ld4(a.trace[k], i0);
                    dst = a.trace[k];
                }
                x.x = x.x * d + s4.x; x.y = x.y * d + s4.y; x.z = x.z * d + s4.z; x.w = x.w * d + s4.w;
                st4(dst, i0, x);
            }
        }
        if (a.i_syn) st4(a.i_syn, i0, make_float4(0.f, 0.f, 0.f, 0.f));
    }
    // Spike lists: one warp scan of the spike counts serves every list, and
    // lane 31 issues all the warp's list reservations at once, so a warp
    // with spikes waits for one atomic round trip, overlapped with the
    // updates of its neurons' spike records.
    int cnt = 0;
#pragma unroll
    for (int k = 0; k < 4 * G; ++k) cnt += sp[k];
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    const int tot = __shfl_sync(0xffffffffu, incl, 31);
    int* list_ids = nullptr;
    int* list_count = nullptr;
    int list_cap = 0x7fffffff;
    if (a.send_hdr) {
        // window send buffer: ids in step order, the running total in send_hdr[win]
        list_ids = a.send_ids;
        list_count = a.send_hdr + a.win;
        list_cap = a.send_cap;
    } else if (a.spike_ids) {
        list_ids = a.spike_ids;
        list_count = a.spike_count;
        if (a.hist_depth > 0) {
            const int slot = static_cast<int>(step % a.hist_depth);
            list_ids += static_cast<long long>(slot) * a.hist_cap;
            list_count += slot;
        }
    }
    int base = 0;
    unsigned long long rbase = 0;
    if (lane == 31 && tot > 0) {
        if (list_count) base = atomicAdd(list_count, tot);
        if (a.send_hdr) atomicAdd(a.send_hdr + static_cast<int>(step % a.win), tot);
        if (a.raster_gid) rbase = atomicAdd(a.raster_count, static_cast<unsigned long long>(tot));
    }
    if (cnt > 0) {
#pragma unroll
        for (int k = 0; k < 4 * G; ++k) {
            if (!sp[k]) continue;
            const int i = ib + (k / 4) * stride + (k % 4);
            if (a.post_recent != nullptr) {
                const int t = static_cast<int>(step);
                const int4 r = a.post_recent[i];
                a.post_recent[i] = make_int4(t, r.x, r.y, r.z);
                const int c = a.post_cnt[i];
                a.post_ring[static_cast<long long>(i) * a.post_ring_k + (c % a.post_ring_k)] = t;
                a.post_cnt[i] = c + 1;
            }
            if (a.win_mask != nullptr) a.win_mask[i] |= 1u << static_cast<int>(step % a.win);
            if (a.spike_stats != nullptr) record_spike_stat(a.spike_stats, i, static_cast<int>(step));
        }
    }
    base = __shfl_sync(0xffffffffu, base, 31);
    rbase = __shfl_sync(0xffffffffu, rbase, 31);
    if (cnt > 0) {
        int pos = base + incl - cnt;
        unsigned long long rpos = rbase + static_cast<unsigned long long>(incl - cnt);
        for (int k = 0; k < 4 * G; ++k) {
            if (!sp[k]) continue;
            const int id = ib + (k / 4) * stride + (k % 4);
            if (list_ids) {
                if (pos < list_cap) list_ids[pos] = a.id_offset + id;
                else if (a.err) atomicCAS(a.err, 0, 4);
            }
            if (a.raster_gid && rpos < static_cast<unsigned long long>(a.raster_cap)) {
                a.raster_step[rpos] = static_cast<int>(step);
                a.raster_gid[rpos] = a.gid_offset + id;
            }
            ++pos;
            ++rpos;
        }
    }
}

// The drive of every neuron of one population for the step (the neuron
// update's own sampler), four neurons a thread: the group of global ids
// 4m .. 4m+3 shares one Philox block.
__global__ void __launch_bounds__(256) drive_fill_kernel(const __grid_constant__ PopArgs a, float* out) {
    long long step = a.step;
    if (a.step_base) step += *a.step_base;
    const long long m0 = a.gid_offset >> 2, m1 = (static_cast<long long>(a.gid_offset) + a.n + 3) >> 2;
    for (long long m = m0 + blockIdx.x * blockDim.x + threadIdx.x; m < m1; m += static_cast<long long>(gridDim.x) * blockDim.x) {
        const float4 x = drive_value4(a, static_cast<uint32_t>(4 * m), static_cast<uint32_t>(step));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const long long i = 4 * m + k - a.gid_offset;
            if (i >= 0 && i < a.n) out[i] = k == 0 ? x.x : k == 1 ? x.y : k == 2 ? x.z : x.w;
        }
    }
}

// The drive of several populations in one launch: block ranges per
// population as in PopGroup, one thread per Philox block (four neurons).
struct DriveGroup {
    PopArgs p[kMaxGroup];
    float* out[kMaxGroup];
    int start[kMaxGroup + 1];
    int n;
};

__global__ void __launch_bounds__(256) drive_fill_group_kernel(const __grid_constant__ DriveGroup g) {
    int q = 0;
    while (q + 1 < g.n && static_cast<int>(blockIdx.x) >= g.start[q + 1]) ++q;
    const PopArgs& a = g.p[q];
    long long step = a.step;
    if (a.step_base) step += *a.step_base;
    const long long m0 = a.gid_offset >> 2, m1 = (static_cast<long long>(a.gid_offset) + a.n + 3) >> 2;
    const long long m = m0 + static_cast<long long>(blockIdx.x - g.start[q]) * blockDim.x + threadIdx.x;
    if (m >= m1) return;
    const float4 x = drive_value4(a, static_cast<uint32_t>(4 * m), static_cast<uint32_t>(step));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const long long i = 4 * m + k - a.gid_offset;
        if (i >= 0 && i < a.n) g.out[q][i] = k == 0 ? x.x : k == 1 ? x.y : k == 2 ? x.z : x.w;
    }
}

template <int MODEL, bool HET, bool COND>
void launch_kind(const PopGroup& g, cudaStream_t s) {
    if (g.n == 1) pop_step_kernel<MODEL, HET, COND><<<g.start[1], kPopThreads, 0, s>>>(g.p[0]);
    else pop_group_kernel<MODEL, HET, COND><<<g.start[g.n], kPopThreads, 0, s>>>(g);
}

// The four-neurons-a-thread LIF kernel applies when every population's
// size is a multiple of 4 and its arrays are 16-byte aligned.
bool lif4_ok(const PopGroup& g) {
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    for (int k = 0; k < g.n; ++k) {
        const PopArgs& a = g.p[k];
        if (a.n % 4 != 0 || !al(a.v) || !al(a.ref) || !al(a.spike) || !al(a.i_syn) || !al(a.drive_values) ||
            a.n_chan > 0)
            return false;
        for (int t = 0; t < a.n_traces; ++t)
            if (!al(a.trace[t]) || !al(a.trace_ring[t])) return false;
    }
    return true;
}

void launch_group(const PopGroup& g, int model, bool het, bool cond, cudaStream_t s) {
    switch (model) {
        case NRN_MODEL_LIF:
            het ? launch_kind<NRN_MODEL_LIF, true, false>(g, s) : launch_kind<NRN_MODEL_LIF, false, false>(g, s);
            break;
        case NRN_MODEL_ADEX:
            if (het) cond ? launch_kind<NRN_MODEL_ADEX, true, true>(g, s) : launch_kind<NRN_MODEL_ADEX, true, false>(g, s);
            else cond ? launch_kind<NRN_MODEL_ADEX, false, true>(g, s) : launch_kind<NRN_MODEL_ADEX, false, false>(g, s);
            break;
        default:
            het ? launch_kind<NRN_MODEL_IZH, true, false>(g, s) : launch_kind<NRN_MODEL_IZH, false, false>(g, s);
            break;
    }
}

}  // namespace
}  // namespace nrn

namespace nrn {
namespace {

// Checks one population's arguments and converts them for the kernel.
nrn_status_t make_args(const nrn_pop_step_t& d, PopArgs& a, bool& het, bool& cond) {
    NRN_CHECK_ARG(d.model >= NRN_MODEL_LIF && d.model <= NRN_MODEL_IZH, "nrn_cuda_pop_step: unknown model");
    NRN_CHECK_ARG(d.n >= 0, "nrn_cuda_pop_step: neuron count must be >= 0");
    if (d.n == 0) return NRN_OK;
    NRN_CHECK_ARG(d.v != nullptr, "nrn_cuda_pop_step: v is required");
    NRN_CHECK_ARG(d.model == NRN_MODEL_LIF || d.aux != nullptr, "nrn_cuda_pop_step: aux (w/u) is required");
    NRN_CHECK_ARG(d.model == NRN_MODEL_IZH || d.refractory != nullptr,
                  "nrn_cuda_pop_step: refractory is required");
    NRN_CHECK_ARG(d.dt >= 0.0, "nrn_cuda_pop_step: dt must be >= 0");
    NRN_CHECK_ARG(d.spike_ids == nullptr || d.spike_count != nullptr,
                  "nrn_cuda_pop_step: spike_ids needs spike_count");
    NRN_CHECK_ARG(d.raster_gid == nullptr || (d.raster_step && d.raster_count),
                  "nrn_cuda_pop_step: raster needs step and count arrays");
    NRN_CHECK_ARG(d.drive.kind >= NRN_DRIVE_NONE && d.drive.kind <= NRN_DRIVE_POISSON_GEXC,
                  "nrn_cuda_pop_step: unknown drive kind");
    cond = d.gin_exc != nullptr;
    NRN_CHECK_ARG(!cond || (d.model == NRN_MODEL_ADEX && d.g_exc && d.g_inh && d.gin_inh),
                  "nrn_cuda_pop_step: conductance input needs an AdEx population and all four arrays");
    NRN_CHECK_ARG(d.drive.kind != NRN_DRIVE_POISSON_GEXC || cond,
                  "nrn_cuda_pop_step: conductance drive needs conductance input");
    a = PopArgs{};
    a.n = d.n;
    a.gid_offset = d.gid_offset;
    a.dtf = static_cast<float>(d.dt);
    const double dt_ms = d.dt * 1000.0;
    a.half = static_cast<float>(0.5 * dt_ms);
    a.dtm = static_cast<float>(dt_ms);
    if (cond) {
        NRN_CHECK_ARG(d.tau_syn_exc > 0.0f && d.tau_syn_inh > 0.0f, "nrn_cuda_pop_step: tau_syn must be > 0");
        a.dec_e = static_cast<float>(std::exp(-d.dt / static_cast<double>(d.tau_syn_exc)));
        a.dec_i = static_cast<float>(std::exp(-d.dt / static_cast<double>(d.tau_syn_inh)));
    }
    a.e_exc = d.e_exc;
    a.e_inh = d.e_inh;
    a.v = d.v; a.aux = d.aux; a.ref = d.refractory; a.spike = d.spike; a.i_syn = d.i_syn;
    a.g_exc = d.g_exc; a.g_inh = d.g_inh; a.gin_exc = d.gin_exc; a.gin_inh = d.gin_inh;
    het = false;
    for (int k = 0; k < NRN_MAX_PARAMS; ++k) {
        a.param[k] = d.param[k];
        a.uniform[k] = d.uniform[k];
        het = het || d.param[k] != nullptr;
    }
    a.drive_kind = d.drive.kind;
    a.d0 = d.drive.p0;
    a.d1 = d.drive.p1;
    a.d_exp = static_cast<float>(std::exp(-static_cast<double>(d.drive.p0)));
    a.n_cdf = 0;
    if (d.drive.kind == NRN_DRIVE_POISSON_CURRENT || d.drive.kind == NRN_DRIVE_POISSON_GEXC) {
        // host float arithmetic, one rounding per operation (no contraction
        // is possible: a product then a quotient, and separate sums)
        volatile float p = a.d_exp, F = p;
        a.cdf[0] = F;
        a.n_cdf = 1;
        for (int k = 1; k < 32; ++k) {
            const float pl = p * a.d0;
            p = pl / static_cast<float>(k);
            F = F + p;
            a.cdf[k] = F;
            a.n_cdf = k + 1;
        }
    }
    a.seed = d.drive.seed;
    a.step = d.step;
    a.step_base = d.step_base;
    a.spike_ids = d.spike_ids;
    a.spike_count = d.spike_count;
    NRN_CHECK_ARG(d.hist_depth <= 0 || d.hist_cap >= d.n, "nrn_cuda_pop_step: history capacity below n");
    a.hist_depth = d.hist_depth;
    a.hist_cap = d.hist_cap;
    a.raster_step = d.raster_step;
    a.raster_gid = d.raster_gid;
    a.raster_count = d.raster_count;
    a.raster_cap = d.raster_cap;
    NRN_CHECK_ARG(d.n_traces >= 0 && d.n_traces <= NRN_MAX_TRACES, "nrn_cuda_pop_step: too many traces");
    a.n_traces = d.n_traces;
    a.trace_slow_ratio = d.trace_slow_ratio;
    a.trace_ring_depth = d.trace_ring_depth;
    NRN_CHECK_ARG(d.trace_ring_depth <= 0 || (d.trace_ring_depth & (d.trace_ring_depth - 1)) == 0,
                  "nrn_cuda_pop_step: trace ring depth must be a power of two");
    for (int k = 0; k < d.n_traces; ++k) {
        NRN_CHECK_ARG(d.trace[k] != nullptr || (d.trace_ring[k] != nullptr && d.trace_ring_depth > 0),
                      "nrn_cuda_pop_step: null trace array");
        a.trace[k] = d.trace[k];
        a.trace_ring[k] = d.trace_ring[k];
        a.trace_decay[k] = d.trace_decay[k];
    }
    a.post_recent = reinterpret_cast<int4*>(d.post_recent);
    a.post_ring = d.post_ring;
    a.post_cnt = d.post_cnt;
    a.post_ring_k = d.post_ring_k;
    NRN_CHECK_ARG(d.post_recent == nullptr || (d.post_ring && d.post_cnt && d.post_ring_k > 0),
                  "nrn_cuda_pop_step: spike history needs ring, count and depth");
    NRN_CHECK_ARG(d.post_recent == nullptr || (reinterpret_cast<uintptr_t>(d.post_recent) % 16) == 0,
                  "nrn_cuda_pop_step: post_recent must be 16-byte aligned");
    a.id_offset = d.id_offset;
    a.win = d.win > 0 ? d.win : 1;
    NRN_CHECK_ARG(a.win <= 32, "nrn_cuda_pop_step: windows are at most 32 steps");
    a.win_mask = d.win > 0 ? d.win_mask : nullptr;
    a.send_hdr = d.win > 0 ? d.send_hdr : nullptr;
    a.send_ids = d.send_ids;
    a.send_cap = d.send_cap;
    a.err = d.err;
    a.drive_values = d.drive_values;
    a.spike_stats = d.spike_stats;
    NRN_CHECK_ARG(d.n_chan >= 0 && d.n_chan <= NRN_MAX_CHANNELS, "nrn_cuda_pop_step: at most 4 synapse channels");
    a.n_chan = d.n_chan;
    for (int c = 0; c < d.n_chan; ++c) {
        const int k = d.chan_kind[c];
        NRN_CHECK_ARG(k >= NRN_SYN_EXP && k <= NRN_SYN_AMPA, "nrn_cuda_pop_step: unknown synapse channel kind");
        NRN_CHECK_ARG(d.chan_in[c] && d.chan_s[c] && (k == NRN_SYN_EXP || d.chan_r[c]),
                      "nrn_cuda_pop_step: null synapse channel array");
        NRN_CHECK_ARG(d.chan_tau_decay[c] > 0.0 && (k == NRN_SYN_EXP || d.chan_tau_rise[c] > 0.0),
                      "nrn_cuda_pop_step: synapse time constants must be > 0");
        a.chan_kind[c] = k;
        a.chan_dec_decay[c] = static_cast<float>(std::exp(-d.dt / d.chan_tau_decay[c]));
        a.chan_dec_rise[c] = k == NRN_SYN_EXP ? 1.0f : static_cast<float>(std::exp(-d.dt / d.chan_tau_rise[c]));
        a.chan_e_rev[c] = d.chan_e_rev[c];
        a.chan_in[c] = d.chan_in[c];
        a.chan_s[c] = d.chan_s[c];
        a.chan_r[c] = d.chan_r[c];
    }
    NRN_CHECK_ARG(a.send_hdr == nullptr || (d.send_ids != nullptr && d.send_cap >= 0),
                  "nrn_cuda_pop_step: send buffer without ids");
    if (d.model != NRN_MODEL_ADEX) cond = false;
    return NRN_OK;
}

}  // namespace

nrn_status_t pop_step_group(const nrn_pop_step_t* list, int n, cudaStream_t s) {
    NRN_CHECK_ARG(n >= 0 && (n == 0 || list != nullptr), "pop_step_group: bad arguments");
    std::vector<char> done(static_cast<size_t>(n), 0);
    for (int q = 0; q < n; ++q) {
        if (done[q]) continue;
        PopGroup g{};
        bool het = false, cond = false;
        NRN_TRY(make_args(list[q], g.p[0], het, cond));
        done[q] = 1;
        if (list[q].n == 0) continue;
        g.n = 1;
        g.start[1] = (list[q].n + kPopThreads - 1) / kPopThreads;
        // later populations of the same kind join this launch
        for (int r = q + 1; r < n && g.n < kMaxGroup; ++r) {
            if (done[r] || list[r].n == 0 || list[r].model != list[q].model) continue;
            PopArgs x;
            bool h2 = false, c2 = false;
            NRN_TRY(make_args(list[r], x, h2, c2));
            if (h2 != het || c2 != cond) continue;
            g.p[g.n] = x;
            g.start[g.n + 1] = g.start[g.n] + (list[r].n + kPopThreads - 1) / kPopThreads;
            ++g.n;
            done[r] = 1;
        }
        if (list[q].model == NRN_MODEL_LIF && !het && lif4_ok(g)) {
            // one group of four neurons a thread: block ranges in units of
            // 4 * kPopThreads neurons (two groups a thread measured slower:
            // 18.6 against 17.3 us per step at 1M neurons)
            constexpr int kGroups = 1;
            int b = 0;
            for (int k = 0; k < g.n; ++k) {
                g.start[k] = b;
                b += (g.p[k].n + 4 * kGroups * kPopThreads - 1) / (4 * kGroups * kPopThreads);
            }
            g.start[g.n] = b;
            lif4_group_kernel<kGroups><<<b, kPopThreads, 0, s>>>(g);
        } else {
            launch_group(g, list[q].model, het, cond, s);
        }
        NRN_CUDA_TRY(cudaGetLastError());
    }
    return NRN_OK;
}

nrn_status_t drive_fill_group(const nrn_pop_step_t* list, float* const* out, int n, cudaStream_t s) {
    for (int q0 = 0; q0 < n; q0 += kMaxGroup) {
        DriveGroup g{};
        int b = 0;
        for (int q = q0; q < n && g.n < kMaxGroup; ++q) {
            bool het = false, cond = false;
            NRN_TRY(make_args(list[q], g.p[g.n], het, cond));
            NRN_CHECK_ARG(out[q] != nullptr || list[q].n == 0, "drive fill: null output");
            if (list[q].n == 0 || g.p[g.n].drive_kind == NRN_DRIVE_NONE) continue;
            g.out[g.n] = out[q];
            g.start[g.n] = b;
            const long long groups = ((static_cast<long long>(list[q].gid_offset) + list[q].n + 3) >> 2) -
                                     (list[q].gid_offset >> 2);
            b += static_cast<int>((groups + 255) / 256);
            ++g.n;
        }
        g.start[g.n] = b;
        if (g.n == 0) continue;
        drive_fill_group_kernel<<<b, 256, 0, s>>>(g);
        NRN_CUDA_TRY(cudaGetLastError());
    }
    return NRN_OK;
}

}  // namespace nrn

extern "C" nrn_status_t nrn_cuda_drive_fill(const nrn_pop_step_t* in, float* out, nrn_stream_t stream) {
    using namespace nrn;
    NRN_CHECK_ARG(in != nullptr && (out != nullptr || in->n == 0), "nrn_cuda_drive_fill: null arguments");
    PopArgs a;
    bool het = false, cond = false;
    NRN_TRY(make_args(*in, a, het, cond));
    if (in->n == 0 || a.drive_kind == NRN_DRIVE_NONE) return NRN_OK;
    const int blocks = std::min((in->n / 4 + 256) / 256, 8 * sm_count_current());
    drive_fill_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a, out);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

extern "C" nrn_status_t nrn_cuda_pop_step(const nrn_pop_step_t* in, nrn_stream_t stream) {
    NRN_CHECK_ARG(in != nullptr, "nrn_cuda_pop_step: null arguments");
    return nrn::pop_step_group(in, 1, reinterpret_cast<cudaStream_t>(stream));
}
