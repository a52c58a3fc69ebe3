// blockdense.cu -- kernels on the API's block-dense connectivity layout.
//
// The nrn:: API exposes connectivity as dense B x B blocks indexed by a CSR
// over target block rows (ConnectivityTensor).  sim_run compiles it into the
// engine's per-synapse CSR; these kernels serve the direct calls:
//   connection_deliver (src/connectivity/connect.cpp:36-79): one warp per
//     target neuron walks the blocks of its block row in CSR order and adds
//     each block's dot product (W * Ms * Mm) . spikes to I_syn;
//   stdp_update (src/plasticity/stdp.cpp:43-141): one thread per synapse
//     entry of the valid (unpadded) part of every block, with the
//     reference's per-synapse traces and clamp.
// plus compaction of a dense spike vector and small gathers/scatters.
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace nrn {
namespace {

__global__ void block_deliver_kernel(const int32_t* row_ptr, const int32_t* col_idx, const float* W, const float* Ms,
                                     const float* Mm, int B, int64_t n_src, int64_t n_tgt, const float* spikes,
                                     float* I) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t n_warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t t = warp; t < n_tgt; t += n_warps) {
        const int64_t tr = t / B, tl = t - tr * B;
        const int32_t b0 = row_ptr[tr], b1 = row_ptr[tr + 1];
        if (b0 == b1) continue;
        float cur = I[t];   // I += block_1 . s; I += block_2 . s; ... in CSR order
        for (int32_t b = b0; b < b1; ++b) {
            const int64_t s0 = static_cast<int64_t>(col_idx[b]) * B;
            const int64_t s_size = (n_src - s0 < B) ? n_src - s0 : B;
            const size_t rowoff = (static_cast<size_t>(b) * B + tl) * B;
            float dot = 0.0f;
            for (int64_t s = lane; s < s_size; s += 32) {
                const float w = (W[rowoff + s] * Ms[rowoff + s]) * Mm[rowoff + s];
                dot += w * spikes[s0 + s];
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            cur = cur + dot;
        }
        if (lane == 0) I[t] = cur;
    }
}

struct BlockStdpArgs {
    const int32_t* row_ptr;
    const int32_t* col_idx;
    float* W;
    const float* Ms;
    const float* Mm;
    float* tp;
    float* tq;
    const float* pre;
    const float* post;
    int B;
    int64_t n_src, n_tgt, n_blocks;
    float decay_pre, decay_post, a_plus, a_minus, lr, w_min, w_max;
};

// Entry (b, r, c) of block b; the block's target row comes from a binary
// search of row_ptr.
__global__ void block_stdp_kernel(const BlockStdpArgs a) {
    const int64_t per_block = static_cast<int64_t>(a.B) * a.B;
    const int64_t total = a.n_blocks * per_block;
    const int64_t n_rows = (a.n_tgt + a.B - 1) / a.B;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = e / per_block;
        const int64_t rc = e - b * per_block;
        const int64_t r = rc / a.B, c = rc - r * a.B;
        int64_t lo = 0, hi = n_rows - 1;
        while (lo < hi) {
            const int64_t mid = (lo + hi + 1) >> 1;
            if (a.row_ptr[mid] <= b) lo = mid; else hi = mid - 1;
        }
        const int64_t t = lo * a.B + r;
        const int64_t s = static_cast<int64_t>(a.col_idx[b]) * a.B + c;
        if (t >= a.n_tgt || s >= a.n_src) continue;   // padding: untouched, as in the reference
        const float pr = a.pre[s], po = a.post[t];
        const float tp = a.tp[e] * a.decay_pre + pr;
        const float tq = a.tq[e] * a.decay_post + po;
        a.tp[e] = tp;
        a.tq[e] = tq;
        const float dw = (a.a_plus * tp) * po - (a.a_minus * tq) * pr;
        float w = a.W[e] + ((dw * a.lr) * a.Ms[e]) * a.Mm[e];
        w = fminf(fmaxf(w, a.w_min), a.w_max);
        a.W[e] = w;
    }
}

__global__ void compact_kernel(const float* x, int64_t n, int32_t* ids, int32_t* count) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const bool hit = i < n && x[i] != 0.0f;
    const unsigned mask = __ballot_sync(0xffffffffu, hit);
    if (mask) {
        const int lane = threadIdx.x & 31;
        const int leader = __ffs(mask) - 1;
        int base = 0;
        if (lane == leader) base = atomicAdd(count, __popc(mask));
        base = __shfl_sync(0xffffffffu, base, leader);
        if (hit) ids[base + __popc(mask & ((1u << lane) - 1u))] = static_cast<int32_t>(i);
    }
}

__global__ void gather_ring_kernel(const float* ring, int64_t n, int64_t depth, int64_t write_pos,
                                   const int64_t* delays, float* out) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t d = delays[i];
        const int64_t row = ((write_pos - d) % depth + depth) % depth;
        out[i] = ring[row * n + i];
    }
}

__global__ void scatter_kernel(const float* src, const int64_t* pos, int64_t n, float* dst) {
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[pos[k]] = src[k];
}

int grid(int64_t n, int threads = 256) {
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, 32 * sm_count_current())));
}

}  // namespace
}  // namespace nrn

extern "C" nrn_status_t nrn_cuda_block_deliver(const nrn_block_csr_t* c, const float* spikes, float* i_syn,
                                               nrn_stream_t stream) {
    using namespace nrn;
    NRN_CHECK_ARG(c && spikes && i_syn, "nrn_cuda_block_deliver: null argument");
    NRN_CHECK_ARG(c->block_size > 0 && c->row_ptr && (c->n_blocks == 0 || (c->col_idx && c->weights &&
                  c->structural_mask && c->modulatory_mask)), "nrn_cuda_block_deliver: bad connectivity");
    if (c->n_target == 0) return NRN_OK;
    const int64_t threads = 256;
    const int64_t blocks = std::min<int64_t>((c->n_target * 32 + threads - 1) / threads, 64 * sm_count_current());
    block_deliver_kernel<<<static_cast<int>(blocks), threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        c->row_ptr, c->col_idx, c->weights, c->structural_mask, c->modulatory_mask, static_cast<int>(c->block_size),
        c->n_source, c->n_target, spikes, i_syn);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

extern "C" nrn_status_t nrn_cuda_block_stdp(const nrn_block_csr_t* c, float* weights, float* trace_pre,
                                            float* trace_post, const float* pre_spikes, const float* post_spikes,
                                            const float* params, nrn_stream_t stream) {
    using namespace nrn;
    NRN_CHECK_ARG(c && weights && trace_pre && trace_post && pre_spikes && post_spikes && params,
                  "nrn_cuda_block_stdp: null argument");
    if (c->n_blocks == 0) return NRN_OK;
    BlockStdpArgs a{};
    a.row_ptr = c->row_ptr;
    a.col_idx = c->col_idx;
    a.W = weights;
    a.Ms = c->structural_mask;
    a.Mm = c->modulatory_mask;
    a.tp = trace_pre;
    a.tq = trace_post;
    a.pre = pre_spikes;
    a.post = post_spikes;
    a.B = static_cast<int>(c->block_size);
    a.n_src = c->n_source;
    a.n_tgt = c->n_target;
    a.n_blocks = c->n_blocks;
    a.decay_pre = params[0];
    a.decay_post = params[1];
    a.a_plus = params[2];
    a.a_minus = params[3];
    a.lr = params[4];
    a.w_min = params[5];
    a.w_max = params[6];
    const int64_t total = c->n_blocks * c->block_size * c->block_size;
    block_stdp_kernel<<<grid(total), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

extern "C" nrn_status_t nrn_cuda_compact(const float* x, int64_t n, int32_t* ids, int32_t* count,
                                         nrn_stream_t stream) {
    using namespace nrn;
    NRN_CHECK_ARG(n >= 0 && n < (int64_t(1) << 31), "nrn_cuda_compact: bad size");
    NRN_CHECK_ARG(n == 0 || (x && ids && count), "nrn_cuda_compact: null argument");
    if (n == 0) return NRN_OK;
    compact_kernel<<<static_cast<int>((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, n, ids,
                                                                                                        count);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

extern "C" nrn_status_t nrn_cuda_gather_ring(const float* ring, int64_t n, int64_t depth, int64_t write_pos,
                                             const int64_t* delays, float* out, nrn_stream_t stream) {
    using namespace nrn;
    NRN_CHECK_ARG(n >= 0 && depth > 0, "nrn_cuda_gather_ring: bad size");
    if (n == 0) return NRN_OK;
    gather_ring_kernel<<<grid(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(ring, n, depth, write_pos, delays,
                                                                                 out);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

extern "C" nrn_status_t nrn_cuda_scatter(const float* src, const int64_t* pos, int64_t n, float* dst,
                                         nrn_stream_t stream) {
    using namespace nrn;
    NRN_CHECK_ARG(n >= 0, "nrn_cuda_scatter: bad size");
    if (n == 0) return NRN_OK;
    scatter_kernel<<<grid(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(src, pos, n, dst);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}
