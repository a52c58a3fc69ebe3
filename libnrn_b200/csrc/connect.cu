// connect.cu -- projections on the device: fixed-degree generation and the
// source-major CSR segmented by delay.
//
// The reference builds Erdos-Renyi block-dense connectivity on the host
// (src/connectivity/topology/random.cpp:25-95) and multiplies every block
// each step.  Here a projection is a synapse list sorted by (source, delay)
// with a stable radix sort, so that one spike's delay-d synapses are one
// contiguous segment; a second stable sort by target gives the
// target-major index that plasticity needs.  Generation uses the same
// Philox draws as the oracle's generator: synapse (row r, slot k) of
// generator `id` comes from Philox(seed; row gid, k, id, 0x434F4E4E).
#include <cuda_runtime.h>

#include <algorithm>
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include "common.cuh"
#include "internal.h"
#include "detmath.cuh"
#include "rng.cuh"

namespace nrn {
namespace {

template <typename T>
nrn_status_t dalloc(T** p, size_t n) {
    if (n == 0) n = 1;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(NRN_ERR_OOM, "device allocation of " + std::to_string(n * sizeof(T)) + " bytes failed");
    }
    return NRN_OK;
}

template <typename T>
void dfree(T*& p) {
    if (p) cudaFree(p);
    p = nullptr;
}

int grid_for(int64_t n, int threads = 256) {
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, 32 * sm_count_current())));
}

__global__ void make_keys(const int32_t* src, const int32_t* tgt, const uint8_t* delay, int64_t n, int32_t n_src,
                          int32_t n_tgt, int32_t dmin, int32_t nd, uint32_t* keys, uint32_t* idx, int* bad) {
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int32_t s = src[k];
        uint32_t key = 0xFFFFFFFFu;
        if (s >= 0) {
            const int32_t t = tgt[k];
            const int32_t dk = static_cast<int32_t>(delay[k]) - dmin;
            if (s >= n_src || t < 0 || t >= n_tgt || dk < 0 || dk >= nd) atomicExch(bad, 1);
            else key = static_cast<uint32_t>(s) * static_cast<uint32_t>(nd) + static_cast<uint32_t>(dk);
        }
        keys[k] = key;
        idx[k] = static_cast<uint32_t>(k);
    }
}

__global__ void count_keys(const uint32_t* keys, int64_t n, uint32_t nkeys, int64_t* counts) {
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint32_t key = keys[k];
        if (key < nkeys) atomicAdd(reinterpret_cast<unsigned long long*>(counts + key), 1ull);
    }
}

__global__ void max_count(const int64_t* counts, int64_t n, unsigned long long* out) {
    unsigned long long m = 0;
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x)
        m = max(m, static_cast<unsigned long long>(counts[k]));
    atomicMax(out, m);
}

__global__ void max_row_len(const int64_t* seg_ptr, int32_t n_src, int32_t nd, unsigned long long* out) {
    unsigned long long m = 0;
    for (int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < n_src;
         j += static_cast<int64_t>(gridDim.x) * blockDim.x)
        m = max(m, static_cast<unsigned long long>(seg_ptr[(j + 1) * nd] - seg_ptr[j * nd]));
    atomicMax(out, m);
}

__global__ void gather_syn(const uint32_t* perm, int64_t n, const int32_t* tgt, const float* w, const float* mod,
                           uint32_t* tgt_o, float* w_o, float* mod_o, int64_t* orig_o) {
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint32_t p = perm[k];
        tgt_o[k] = static_cast<uint32_t>(tgt[p]);
        w_o[k] = w[p];
        if (mod_o) mod_o[k] = mod[p];
        if (orig_o) orig_o[k] = p;
    }
}

__global__ void iota_u32(uint32_t* a, int64_t n) {
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x)
        a[k] = static_cast<uint32_t>(k);
}

// Source of every CSR position from seg_ptr: one thread per (source, delay) segment.
__global__ void seg_sources(const int64_t* seg_ptr, int32_t n_src, int32_t nd, uint32_t* src_of) {
    const int64_t nseg = static_cast<int64_t>(n_src) * nd;
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < nseg;
         g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint32_t j = static_cast<uint32_t>(g / nd);
        for (int64_t p = seg_ptr[g]; p < seg_ptr[g + 1]; ++p) src_of[p] = j;
    }
}

__global__ void gather_u32(const uint32_t* perm, int64_t n, const uint32_t* in, uint32_t* out) {
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[k] = in[perm[k]];
}

// Delay (steps) of every CSR position: one thread per (source, delay) segment.
__global__ void seg_delays(const int64_t* seg_ptr, int32_t n_src, int32_t nd, int32_t dmin, uint8_t* delay_of) {
    const int64_t nseg = static_cast<int64_t>(n_src) * nd;
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < nseg;
         g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint8_t d = static_cast<uint8_t>(dmin + static_cast<int32_t>(g % nd));
        for (int64_t p = seg_ptr[g]; p < seg_ptr[g + 1]; ++p) delay_of[p] = d;
    }
}

// Sort keys of the deterministic index: target above the CSR position (the
// CSR is ordered by source, then delay, then the caller's list order).
__global__ void det_keys(const uint32_t* tgt, int64_t n, unsigned long long* key, uint32_t* pos) {
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        key[k] = (static_cast<unsigned long long>(tgt[k]) << 32) | static_cast<unsigned long long>(k);
        pos[k] = static_cast<uint32_t>(k);
    }
}

__global__ void det_targets(const unsigned long long* key, int64_t n, uint32_t* tgt_of) {
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x)
        tgt_of[k] = static_cast<uint32_t>(key[k] >> 32);
}

__global__ void gather_u8(const uint32_t* perm, int64_t n, const uint8_t* in, uint8_t* out) {
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[k] = in[perm[k]];
}

// Raster entries as sort keys: the step above `shift` bits of neuron id.
__global__ void raster_pack(const int32_t* step, const int32_t* gid, int64_t n, int shift, unsigned long long* key) {
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x)
        key[k] = (static_cast<unsigned long long>(static_cast<uint32_t>(step[k])) << shift) |
                 static_cast<uint32_t>(gid[k]);
}

__global__ void raster_unpack(const unsigned long long* key, int64_t n, int shift, int32_t* step, int32_t* gid) {
    const unsigned long long mask = (1ull << shift) - 1;
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        step[k] = static_cast<int32_t>(key[k] >> shift);
        gid[k] = static_cast<int32_t>(key[k] & mask);
    }
}

__global__ void gen_kernel(const GenArgs g, int32_t* src, int32_t* tgt, float* w, uint8_t* delay) {
    const int64_t total = static_cast<int64_t>(g.n_rows) * g.degree;
    const uint32_t span = static_cast<uint32_t>(g.dmax - g.dmin + 1);
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int32_t r = static_cast<int32_t>(e / g.degree);
        const uint32_t k = static_cast<uint32_t>(e - static_cast<int64_t>(r) * g.degree);
        const int32_t gid = g.row_offset + r;
        const bool self = gid >= g.col_offset && gid < g.col_offset + g.col_n;
        const uint32_t m = static_cast<uint32_t>(self ? g.col_n - 1 : g.col_n);
        const U4 x = philox4x32_10(U4{static_cast<uint32_t>(gid), k, g.gen_id, kStreamConn}, g.seed);
        uint32_t c = __umulhi(x.x, m);
        if (self && c >= static_cast<uint32_t>(gid - g.col_offset)) c += 1;
        const uint32_t d = static_cast<uint32_t>(g.dmin) + __umulhi(x.y, span);
        const int32_t src_g = g.out_degree ? gid : g.col_offset + static_cast<int32_t>(c);
        const int32_t tgt_g = g.out_degree ? g.col_offset + static_cast<int32_t>(c) : gid;
        const bool keep = tgt_g >= g.keep_lo && tgt_g < g.keep_hi;
        src[e] = keep ? src_g - g.src_offset : -1;
        tgt[e] = tgt_g - g.keep_lo;
        w[e] = g.w_lo + g.w_span * u01(x.z);
        delay[e] = static_cast<uint8_t>(d);
    }
}

// ---------------------------------------------------------------------------
// Random (Erdos-Renyi) and distance-dependent connectivity, one thread per
// target row.  Rows are this GPU's targets (population indices lo .. lo +
// n_rows); sources are the whole source population.
//   ER: each (source, target) pair with probability p, drawn by geometric
//       skips over the sources: gap = floor(ln u / ln(1 - p)), u from
//       Philox(seed; row gid, draw k, gen, ER stream) word 0;
//   distance-dependent: 1D positions x_s = s L / n_src, x_t = t L / n_tgt
//       (L = max_distance), p = max(exp(-d^2 / 2 sigma^2), p_min); pair
//       (t, s) connected iff word (s % 4) of Philox(seed; row gid, s / 4, gen,
//       distance stream) < floor(p 2^32), sources outside the window where
//       p < 2^-40 skipped.
// Delay and weight of a synapse from Philox(seed; row gid, k, gen, delay
// stream): delay dmin + floor(w0 span / 2^32), weight w_lo + w_span u01(w1),
// k the synapse's rank in its row.  Autapses are skipped when the source and
// target populations are the same.  exp and log are detmath's, so the host
// oracle draws the same synapses.
constexpr uint32_t kStreamEr = 0x45524E44u;
constexpr uint32_t kStreamDist = 0x44495354u;
constexpr uint32_t kStreamSyn = 0x53594E31u;

__device__ __forceinline__ uint32_t prob_threshold(double p) {
    if (!(p > 0.0)) return 0u;
    const double t = floor(p * 4294967296.0);
    return t >= 4294967295.0 ? 0xFFFFFFFFu : static_cast<uint32_t>(t);
}

// Calls emit(source index, rank in row) for the row's synapses in source order.
template <class F>
__device__ void random_row(const RandArgs& a, int32_t r, F&& emit) {
    const int32_t t = a.tgt_lo + r;                                   // target population index
    const uint32_t gid = static_cast<uint32_t>(a.tgt_gid_offset + t);
    const int32_t self = a.same_pop ? t : -1;
    uint32_t k = 0;
    if (a.rule == NRN_GEN_ER) {
        if (a.p <= 0.0) return;
        int64_t pos = -1;
        for (uint32_t draw = 0;; ++draw) {
            int64_t step = 1;
            if (a.p < 1.0) {
                const U4 x = philox4x32_10(U4{gid, draw, a.gen_id, kStreamEr}, a.seed);
                const double u = (static_cast<double>(x.x) + 0.5) * (1.0 / 4294967296.0);
                double l = det_log(u);
                if (l > 0.0) l = 0.0;
                const double gap = floor(l / a.log1mp);
                if (gap >= static_cast<double>(a.n_src)) break;
                step = 1 + static_cast<int64_t>(gap);
            }
            pos += step;
            if (pos >= a.n_src) break;
            if (pos != self) emit(static_cast<int32_t>(pos), k++);
        }
        return;
    }
    // distance-dependent
    const double xt = static_cast<double>(t) * a.spacing_tgt;
    int64_t s0 = 0, s1 = a.n_src;
    if (a.half_window >= 0.0 && a.spacing_src > 0.0) {
        const double lo = floor((xt - a.half_window) / a.spacing_src);
        const double hi = ceil((xt + a.half_window) / a.spacing_src) + 1.0;
        s0 = lo < 0.0 ? 0 : static_cast<int64_t>(lo);
        s1 = hi > static_cast<double>(a.n_src) ? a.n_src : static_cast<int64_t>(hi);
    }
    U4 x{0u, 0u, 0u, 0u};
    for (int64_t s = s0; s < s1; ++s) {
        if ((s & 3) == 0 || s == s0)
            x = philox4x32_10(U4{gid, static_cast<uint32_t>(s >> 2), a.gen_id, kStreamDist}, a.seed);
        if (s == self) continue;
        const double d = xt - static_cast<double>(s) * a.spacing_src;
        double p = det_exp_neg((d * d) * a.inv_two_sigma_sq);
        if (p < a.p_min) p = a.p_min;
        const uint32_t w = (s & 3) == 0 ? x.x : (s & 3) == 1 ? x.y : (s & 3) == 2 ? x.z : x.w;
        if (w < prob_threshold(p)) emit(static_cast<int32_t>(s), k++);
    }
}

__global__ void random_count(const RandArgs a, int64_t* counts) {
    for (int32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < a.n_rows; r += gridDim.x * blockDim.x) {
        int64_t c = 0;
        random_row(a, r, [&](int32_t, uint32_t) { ++c; });
        counts[r] = c;
    }
}

__global__ void random_fill(const RandArgs a, const int64_t* offsets, int32_t* src, int32_t* tgt, float* w,
                            uint8_t* delay) {
    const uint32_t span = static_cast<uint32_t>(a.dmax - a.dmin + 1);
    for (int32_t r = blockIdx.x * blockDim.x + threadIdx.x; r < a.n_rows; r += gridDim.x * blockDim.x) {
        int64_t o = offsets[r];
        const uint32_t gid = static_cast<uint32_t>(a.tgt_gid_offset + a.tgt_lo + r);
        random_row(a, r, [&](int32_t sidx, uint32_t k) {
            const U4 y = philox4x32_10(U4{gid, k, a.gen_id, kStreamSyn}, a.seed);
            src[o] = sidx;
            tgt[o] = r;
            delay[o] = static_cast<uint8_t>(static_cast<uint32_t>(a.dmin) + __umulhi(y.x, span));
            w[o] = a.w_lo + a.w_span * u01(y.y);
            ++o;
        });
    }
}

}  // namespace

nrn_status_t generate_random(const RandArgs& a, DevSynList* out, cudaStream_t s) {
    int64_t* counts = nullptr;
    void* tmp = nullptr;
    size_t tmp_bytes = 0;
    nrn_status_t st = NRN_OK;
    *out = DevSynList{};
    NRN_TRY(dalloc(&counts, static_cast<size_t>(a.n_rows) + 1));
    auto fin = [&](nrn_status_t r) {
        dfree(counts);
        if (tmp) cudaFree(tmp);
        if (r != NRN_OK) out->release();
        return r;
    };
    if (cudaMemsetAsync(counts, 0, (static_cast<size_t>(a.n_rows) + 1) * sizeof(int64_t), s) != cudaSuccess)
        return fin(cuda_fail(cudaGetLastError(), "generator counts"));
    if (a.n_rows > 0) {
        random_count<<<grid_for(a.n_rows, 128), 128, 0, s>>>(a, counts);
        if (cudaGetLastError() != cudaSuccess) return fin(cuda_fail(cudaGetLastError(), "random_count"));
    }
    // exclusive scan in place: counts -> row offsets, counts[n_rows] = total
    if (cub::DeviceScan::ExclusiveSum(nullptr, tmp_bytes, counts, counts, static_cast<int64_t>(a.n_rows) + 1, s) !=
            cudaSuccess ||
        cudaMalloc(&tmp, tmp_bytes) != cudaSuccess ||
        cub::DeviceScan::ExclusiveSum(tmp, tmp_bytes, counts, counts, static_cast<int64_t>(a.n_rows) + 1, s) !=
            cudaSuccess)
        return fin(cuda_fail(cudaGetLastError(), "generator scan"));
    int64_t total = 0;
    if (cudaMemcpyAsync(&total, counts + a.n_rows, sizeof(int64_t), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return fin(cuda_fail(cudaGetLastError(), "generator total"));
    out->n = total;
    if ((st = dalloc(&out->src, total)) != NRN_OK || (st = dalloc(&out->tgt, total)) != NRN_OK ||
        (st = dalloc(&out->w, total)) != NRN_OK || (st = dalloc(&out->delay, total)) != NRN_OK)
        return fin(st);
    if (total > 0 && a.n_rows > 0) {
        random_fill<<<grid_for(a.n_rows, 128), 128, 0, s>>>(a, counts, out->src, out->tgt, out->w, out->delay);
        if (cudaGetLastError() != cudaSuccess) return fin(cuda_fail(cudaGetLastError(), "random_fill"));
    }
    if (cudaStreamSynchronize(s) != cudaSuccess) return fin(cuda_fail(cudaGetLastError(), "generator"));
    return fin(NRN_OK);
}

int sm_count_current() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

void free_csr(DevCsr& c) {
    dfree(c.seg_ptr);
    dfree(c.tgt);
    dfree(c.w);
    dfree(c.mod);
    dfree(c.orig);
    dfree(c.in_ptr);
    dfree(c.in_syn);
    dfree(c.in_src);
    dfree(c.det_ptr);
    dfree(c.det_syn);
    dfree(c.det_src);
    dfree(c.det_delay);
}

nrn_status_t build_det_index(DevCsr& c, cudaStream_t s) {
    const int64_t n = c.nnz;
    unsigned long long *k1 = nullptr, *k2 = nullptr;
    uint32_t *p1 = nullptr, *p2 = nullptr, *src_of = nullptr, *tgt_of = nullptr;
    uint8_t* d_of = nullptr;
    int64_t* counts = nullptr;
    void* tmp = nullptr;
    size_t tmp_bytes = 0;
    nrn_status_t st = NRN_OK;
    auto cleanup = [&]() {
        dfree(k1); dfree(k2); dfree(p1); dfree(p2); dfree(src_of); dfree(tgt_of); dfree(d_of); dfree(counts);
        if (tmp) cudaFree(tmp);
        tmp = nullptr;
    };
#define STEP(x)                       \
    do {                              \
        st = (x);                     \
        if (st != NRN_OK) {           \
            cleanup();                \
            return st;                \
        }                             \
    } while (0)
#define CSTEP(x) STEP(((x) == cudaSuccess) ? NRN_OK : cuda_fail(cudaGetLastError(), #x))
    STEP(dalloc(&k1, n));
    STEP(dalloc(&k2, n));
    STEP(dalloc(&p1, n));
    STEP(dalloc(&p2, n));
    STEP(dalloc(&src_of, n));
    STEP(dalloc(&tgt_of, n));
    STEP(dalloc(&d_of, n));
    STEP(dalloc(&counts, static_cast<size_t>(c.n_tgt) + 1));
    if (n > 0) {
        det_keys<<<grid_for(n), 256, 0, s>>>(c.tgt, n, k1, p1);
        CSTEP(cudaGetLastError());
        seg_sources<<<grid_for(static_cast<int64_t>(c.n_src) * c.nd), 256, 0, s>>>(c.seg_ptr, c.n_src, c.nd, src_of);
        CSTEP(cudaGetLastError());
        seg_delays<<<grid_for(static_cast<int64_t>(c.n_src) * c.nd), 256, 0, s>>>(c.seg_ptr, c.n_src, c.nd, c.dmin,
                                                                                   d_of);
        CSTEP(cudaGetLastError());
    }
    {
        cub::DoubleBuffer<unsigned long long> dk(k1, k2);
        cub::DoubleBuffer<uint32_t> dv(p1, p2);
        CSTEP(cub::DeviceRadixSort::SortPairs(nullptr, tmp_bytes, dk, dv, static_cast<int>(n), 0, 64, s));
        CSTEP(cudaMalloc(&tmp, tmp_bytes));
        CSTEP(cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, dk, dv, static_cast<int>(n), 0, 64, s));
        if (dk.Current() != k1) std::swap(k1, k2);
        if (dv.Current() != p1) std::swap(p1, p2);
        cudaFree(tmp);
        tmp = nullptr;
    }
    CSTEP(cudaMemsetAsync(counts, 0, (static_cast<size_t>(c.n_tgt) + 1) * sizeof(int64_t), s));
    if (n > 0) {
        det_targets<<<grid_for(n), 256, 0, s>>>(k1, n, tgt_of);
        CSTEP(cudaGetLastError());
        count_keys<<<grid_for(n), 256, 0, s>>>(tgt_of, n, static_cast<uint32_t>(c.n_tgt), counts);
        CSTEP(cudaGetLastError());
    }
    STEP(dalloc(&c.det_ptr, static_cast<size_t>(c.n_tgt) + 1));
    tmp_bytes = 0;
    CSTEP(cub::DeviceScan::ExclusiveSum(nullptr, tmp_bytes, counts, c.det_ptr, static_cast<int64_t>(c.n_tgt) + 1, s));
    CSTEP(cudaMalloc(&tmp, tmp_bytes));
    CSTEP(cub::DeviceScan::ExclusiveSum(tmp, tmp_bytes, counts, c.det_ptr, static_cast<int64_t>(c.n_tgt) + 1, s));
    STEP(dalloc(&c.det_syn, n));
    STEP(dalloc(&c.det_src, n));
    STEP(dalloc(&c.det_delay, n));
    CSTEP(cudaMemcpyAsync(c.det_syn, p1, n * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s));
    if (n > 0) {
        gather_u32<<<grid_for(n), 256, 0, s>>>(p1, n, src_of, c.det_src);
        CSTEP(cudaGetLastError());
        gather_u8<<<grid_for(n), 256, 0, s>>>(p1, n, d_of, c.det_delay);
        CSTEP(cudaGetLastError());
    }
    CSTEP(cudaStreamSynchronize(s));
    cleanup();
    return NRN_OK;
#undef CSTEP
#undef STEP
}

nrn_status_t build_csr(DevCsr& c, int32_t n_src, int32_t n_tgt, const int32_t* src, const int32_t* tgt,
                       const float* w, const uint8_t* delay, const float* mod, int64_t n_in, bool keep_orig,
                       cudaStream_t s) {
    NRN_CHECK_ARG(n_in >= 0 && n_in < (int64_t(1) << 32) - 1, "projection too large (2^32 synapses per GPU)");
    NRN_CHECK_ARG(static_cast<uint64_t>(n_src) * c.nd < 0xFFFFFFFFull, "too many (source, delay) segments");
    c.n_src = n_src;
    c.n_tgt = n_tgt;
    const uint32_t nkeys = static_cast<uint32_t>(n_src) * static_cast<uint32_t>(c.nd);
    uint32_t *keys = nullptr, *keys2 = nullptr, *idx = nullptr, *idx2 = nullptr;
    int64_t* counts = nullptr;
    int* bad = nullptr;
    void* tmp = nullptr;
    size_t tmp_bytes = 0;
    nrn_status_t st = NRN_OK;
    int hbad = 0;
    int end_bit = 1;
    while (end_bit < 32 && (uint64_t(1) << end_bit) <= nkeys) ++end_bit;
    auto cleanup = [&]() {
        dfree(keys); dfree(keys2); dfree(idx); dfree(idx2); dfree(counts); dfree(bad);
        if (tmp) cudaFree(tmp);
        tmp = nullptr;
    };
#define STEP(x)                       \
    do {                              \
        st = (x);                     \
        if (st != NRN_OK) {           \
            cleanup();                \
            return st;                \
        }                             \
    } while (0)
#define CSTEP(x) STEP(((x) == cudaSuccess) ? NRN_OK : cuda_fail(cudaGetLastError(), #x))
    STEP(dalloc(&keys, n_in));
    STEP(dalloc(&keys2, n_in));
    STEP(dalloc(&idx, n_in));
    STEP(dalloc(&idx2, n_in));
    STEP(dalloc(&bad, 1));
    STEP(dalloc(&counts, static_cast<size_t>(nkeys) + 1));
    CSTEP(cudaMemsetAsync(bad, 0, sizeof(int), s));
    CSTEP(cudaMemsetAsync(counts, 0, (static_cast<size_t>(nkeys) + 1) * sizeof(int64_t), s));
    if (n_in > 0) {
        make_keys<<<grid_for(n_in), 256, 0, s>>>(src, tgt, delay, n_in, n_src, n_tgt, c.dmin, c.nd, keys, idx, bad);
        CSTEP(cudaGetLastError());
    }
    CSTEP(cudaMemcpyAsync(&hbad, bad, sizeof(int), cudaMemcpyDeviceToHost, s));
    CSTEP(cudaStreamSynchronize(s));
    if (hbad) {
        cleanup();
        return fail(NRN_ERR_INVALID, "projection: source, target or delay out of range");
    }
    // stable sort of positions by (source, delay); dropped entries sort last
    {
        cub::DoubleBuffer<uint32_t> dk(keys, keys2), dv(idx, idx2);
        const int bits = (nkeys > 0 && end_bit < 32) ? end_bit + 1 : 32;   // + the drop sentinel
        CSTEP(cub::DeviceRadixSort::SortPairs(nullptr, tmp_bytes, dk, dv, static_cast<int>(n_in), 0, 32, s));
        CSTEP(cudaMalloc(&tmp, tmp_bytes));
        (void)bits;
        CSTEP(cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, dk, dv, static_cast<int>(n_in), 0, 32, s));
        if (dk.Current() != keys) std::swap(keys, keys2);
        if (dv.Current() != idx) std::swap(idx, idx2);
        cudaFree(tmp);
        tmp = nullptr;
    }
    // segment offsets: exclusive scan of the per-key counts
    if (n_in > 0) {
        count_keys<<<grid_for(n_in), 256, 0, s>>>(keys, n_in, nkeys, counts);
        CSTEP(cudaGetLastError());
    }
    {
        unsigned long long* dm = nullptr;
        unsigned long long hm = 0;
        STEP(dalloc(&dm, 1));
        CSTEP(cudaMemsetAsync(dm, 0, sizeof(*dm), s));
        max_count<<<grid_for(nkeys), 256, 0, s>>>(counts, nkeys, dm);
        CSTEP(cudaMemcpyAsync(&hm, dm, sizeof(hm), cudaMemcpyDeviceToHost, s));
        CSTEP(cudaStreamSynchronize(s));
        dfree(dm);
        c.max_seg = static_cast<int32_t>(hm);
    }
    STEP(dalloc(&c.seg_ptr, static_cast<size_t>(nkeys) + 1));
    tmp_bytes = 0;
    CSTEP(cub::DeviceScan::ExclusiveSum(nullptr, tmp_bytes, counts, c.seg_ptr, static_cast<int64_t>(nkeys) + 1, s));
    CSTEP(cudaMalloc(&tmp, tmp_bytes));
    CSTEP(cub::DeviceScan::ExclusiveSum(tmp, tmp_bytes, counts, c.seg_ptr, static_cast<int64_t>(nkeys) + 1, s));
    {
        unsigned long long* dm = nullptr;
        unsigned long long hm = 0;
        STEP(dalloc(&dm, 1));
        CSTEP(cudaMemsetAsync(dm, 0, sizeof(*dm), s));
        max_row_len<<<grid_for(n_src), 256, 0, s>>>(c.seg_ptr, n_src, c.nd, dm);
        CSTEP(cudaMemcpyAsync(&hm, dm, sizeof(hm), cudaMemcpyDeviceToHost, s));
        CSTEP(cudaStreamSynchronize(s));
        dfree(dm);
        c.max_row = static_cast<int32_t>(hm);
    }
    int64_t nnz = 0;
    CSTEP(cudaMemcpyAsync(&nnz, c.seg_ptr + nkeys, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    CSTEP(cudaStreamSynchronize(s));
    c.nnz = nnz;
    STEP(dalloc(&c.tgt, nnz));
    STEP(dalloc(&c.w, nnz));
    if (mod) STEP(dalloc(&c.mod, nnz));
    if (keep_orig) STEP(dalloc(&c.orig, nnz));
    if (nnz > 0) {
        gather_syn<<<grid_for(nnz), 256, 0, s>>>(idx, nnz, tgt, w, mod, c.tgt, c.w, c.mod, c.orig);
        CSTEP(cudaGetLastError());
    }
    CSTEP(cudaStreamSynchronize(s));
    cleanup();
    return NRN_OK;
#undef CSTEP
#undef STEP
}

nrn_status_t build_transpose(DevCsr& c, cudaStream_t s) {
    const int64_t n = c.nnz;
    uint32_t *keys = nullptr, *keys2 = nullptr, *pos = nullptr, *pos2 = nullptr, *src_of = nullptr;
    int64_t* counts = nullptr;
    void* tmp = nullptr;
    size_t tmp_bytes = 0;
    nrn_status_t st = NRN_OK;
    auto cleanup = [&]() {
        dfree(keys); dfree(keys2); dfree(pos); dfree(pos2); dfree(src_of); dfree(counts);
        if (tmp) cudaFree(tmp);
        tmp = nullptr;
    };
#define STEP(x)                       \
    do {                              \
        st = (x);                     \
        if (st != NRN_OK) {           \
            cleanup();                \
            return st;                \
        }                             \
    } while (0)
#define CSTEP(x) STEP(((x) == cudaSuccess) ? NRN_OK : cuda_fail(cudaGetLastError(), #x))
    STEP(dalloc(&keys, n));
    STEP(dalloc(&keys2, n));
    STEP(dalloc(&pos, n));
    STEP(dalloc(&pos2, n));
    STEP(dalloc(&src_of, n));
    STEP(dalloc(&counts, static_cast<size_t>(c.n_tgt) + 1));
    CSTEP(cudaMemcpyAsync(keys, c.tgt, n * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s));
    if (n > 0) {
        iota_u32<<<grid_for(n), 256, 0, s>>>(pos, n);
        CSTEP(cudaGetLastError());
        seg_sources<<<grid_for(static_cast<int64_t>(c.n_src) * c.nd), 256, 0, s>>>(c.seg_ptr, c.n_src, c.nd, src_of);
        CSTEP(cudaGetLastError());
    }
    {
        cub::DoubleBuffer<uint32_t> dk(keys, keys2), dv(pos, pos2);
        CSTEP(cub::DeviceRadixSort::SortPairs(nullptr, tmp_bytes, dk, dv, static_cast<int>(n), 0, 32, s));
        CSTEP(cudaMalloc(&tmp, tmp_bytes));
        CSTEP(cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, dk, dv, static_cast<int>(n), 0, 32, s));
        if (dk.Current() != keys) std::swap(keys, keys2);
        if (dv.Current() != pos) std::swap(pos, pos2);
        cudaFree(tmp);
        tmp = nullptr;
    }
    CSTEP(cudaMemsetAsync(counts, 0, (static_cast<size_t>(c.n_tgt) + 1) * sizeof(int64_t), s));
    if (n > 0) {
        count_keys<<<grid_for(n), 256, 0, s>>>(keys, n, static_cast<uint32_t>(c.n_tgt), counts);
        CSTEP(cudaGetLastError());
    }
    {
        unsigned long long* dm = nullptr;
        unsigned long long hm = 0;
        STEP(dalloc(&dm, 1));
        CSTEP(cudaMemsetAsync(dm, 0, sizeof(*dm), s));
        max_count<<<grid_for(c.n_tgt), 256, 0, s>>>(counts, c.n_tgt, dm);
        CSTEP(cudaMemcpyAsync(&hm, dm, sizeof(hm), cudaMemcpyDeviceToHost, s));
        CSTEP(cudaStreamSynchronize(s));
        dfree(dm);
        c.max_in = static_cast<int32_t>(hm);
    }
    STEP(dalloc(&c.in_ptr, static_cast<size_t>(c.n_tgt) + 1));
    tmp_bytes = 0;
    CSTEP(cub::DeviceScan::ExclusiveSum(nullptr, tmp_bytes, counts, c.in_ptr, static_cast<int64_t>(c.n_tgt) + 1, s));
    CSTEP(cudaMalloc(&tmp, tmp_bytes));
    CSTEP(cub::DeviceScan::ExclusiveSum(tmp, tmp_bytes, counts, c.in_ptr, static_cast<int64_t>(c.n_tgt) + 1, s));
    STEP(dalloc(&c.in_syn, n));
    STEP(dalloc(&c.in_src, n));
    CSTEP(cudaMemcpyAsync(c.in_syn, pos, n * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s));
    if (n > 0) {
        gather_u32<<<grid_for(n), 256, 0, s>>>(pos, n, src_of, c.in_src);
        CSTEP(cudaGetLastError());
    }
    CSTEP(cudaStreamSynchronize(s));
    cleanup();
    return NRN_OK;
#undef CSTEP
#undef STEP
}

nrn_status_t sort_raster(int32_t* step, int32_t* gid, int64_t n, int gid_bits, int step_bits, RasterSortScratch& sc,
                         cudaStream_t s) {
    if (n <= 1) return NRN_OK;
    NRN_CHECK_ARG(n < (int64_t(1) << 31), "raster too large to sort at once");
    NRN_CHECK_ARG(gid_bits >= 1 && gid_bits <= 32 && step_bits >= 1 && gid_bits + step_bits <= 64,
                  "raster sort: key does not fit 64 bits");
    const int end_bit = gid_bits + step_bits;
    // buffers kept from earlier reads, grown when a read is larger
    if (n > sc.cap) {
        sc.release();
        nrn_status_t st = dalloc(&sc.a, n);
        if (st == NRN_OK) st = dalloc(&sc.b, n);
        if (st != NRN_OK) {
            sc.release();
            return st;
        }
        sc.cap = n;
    }
    cub::DoubleBuffer<unsigned long long> db(sc.a, sc.b);
    size_t need = 0;
    cudaError_t e = cub::DeviceRadixSort::SortKeys(nullptr, need, db, static_cast<int>(n), 0, end_bit, s);
    if (e != cudaSuccess) return cuda_fail(e, "raster sort size");
    if (need > sc.tmp_bytes) {
        if (sc.tmp) cudaFree(sc.tmp);
        sc.tmp = nullptr;
        sc.tmp_bytes = 0;
        e = cudaMalloc(&sc.tmp, need);
        if (e != cudaSuccess) return cuda_fail(e, "raster sort scratch");
        sc.tmp_bytes = need;
    }
    raster_pack<<<grid_for(n), 256, 0, s>>>(step, gid, n, gid_bits, sc.a);
    size_t bytes = sc.tmp_bytes;
    e = cub::DeviceRadixSort::SortKeys(sc.tmp, bytes, db, static_cast<int>(n), 0, end_bit, s);
    if (e == cudaSuccess) {
        raster_unpack<<<grid_for(n), 256, 0, s>>>(db.Current(), n, gid_bits, step, gid);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) return cuda_fail(e, "raster sort");
    return NRN_OK;
}

nrn_status_t generate(const GenArgs& g, int32_t* src, int32_t* tgt, float* w, uint8_t* delay, cudaStream_t s) {
    const int64_t total = static_cast<int64_t>(g.n_rows) * g.degree;
    if (total == 0) return NRN_OK;
    gen_kernel<<<grid_for(total), 256, 0, s>>>(g, src, tgt, w, delay);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

}  // namespace nrn
