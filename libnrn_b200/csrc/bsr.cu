// bsr.cu -- batched block-sparse synaptic propagation on the tensor cores.
//
// For B = 64 independent trials, one step computes
//     I[post, trial] += sum over blocks (r, c) of W[r,c] (64x64) . S[c-block, trial]
// the reference's intended block-dense product (synaptic_current_block_dense_
// kernel, src/synapse/kernels/synapse_kernels.cu:8-30; an empty stub there)
// batched over trials, so each block is a dense 64x64x64 contraction:
// bf16 weights and 0/1 spikes, fp32 accumulation.
//
// Layout.  Every 64x64 bf16 operand tile (a weight block: rows = post, K =
// pre; a spike tile of pre block c: rows = trial, K = pre) is stored in HBM
// already in the tensor core's K-major canonical order without swizzle:
// element (row, k) at (row/8)*512 + (k/8)*64 + (row%8)*8 + k%8 (bf16
// units), i.e. 8x8 core matrices of 128 contiguous bytes, the eight K
// groups of an 8-row group 128 B apart (leading offset) and 8-row groups
// 1 KB apart (stride offset).  A tile is then one contiguous 8 KB copy.
//
// Kernel (persistent, one CTA per SM, 6 warps):
//   warp 0   producer: for each block of its block rows, waits for a free
//            stage, then two 8 KB bulk copies (weights, spike tile) into
//            the stage, completing on the stage's mbarrier;
//   warp 1   issuer (one thread): per block four tcgen05.mma (M=64, N=64,
//            K=16, bf16 -> fp32) into one of two TMEM accumulators, then
//            tcgen05.commit frees the stage; after a row's last block the
//            commit hands the accumulator to the epilogue;
//   warps 2-5 epilogue: tcgen05.ld of the 64x64 fp32 accumulator (TMEM
//            lanes of the warp's sub-partition), release of the
//            accumulator, then I += D (each thread one post neuron, 64
//            trials = 256 contiguous bytes).
// Every wait is bounded: on a timeout the CTA raises an error flag, lets
// the other roles stop, waits for its own copies and MMAs, frees its TMEM
// and returns.
//
// Bound: HBM.  Per block 8 KB of weights are read once per step (the spike
// tiles, 32 MB for 262,144 pre neurons, stay in L2), against 2*64^3 flops:
// 64 flops per weight byte, below the ridge of ~290.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "internal.h"
#include "rng.cuh"

namespace nrn {
namespace {

constexpr int kMaxStages = 13;   // 13 x 16 KB: the most one CTA's shared memory holds
constexpr int kTileElems = 4096;
constexpr int kTileBytes = 8192;
constexpr int kBsrThreads = 192;
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr uint32_t kStreamBsr = 0x42535250u;

enum { ERR_BSR_TIMEOUT = 5 };

struct BsrArgs {
    int32_t n_rows;
    int32_t stages;   // pipeline stages of 16 KB (weights + spikes), <= kMaxStages
    const int32_t* row_ptr;
    const int32_t* col_idx;
    const uint16_t* tiles;
    const uint16_t* spikes;
    float* i_syn;
    int* err;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase of `parity` to complete; false on timeout or abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    for (uint32_t k = 0; k < kSpinLimit; ++k) {
        if (mbar_try_wait(bar, parity)) return true;
        if (abort && *abort) return false;
    }
    return false;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// L2 policies: the weights stream through once per step (evict first); the
// spike tiles are read by every block of their column (evict last).
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Plain (untiled, no multicast) bulk copy global -> this CTA's shared memory.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, no swizzle: leading offset 128 B (next 8-element K group), stride
// offset 1 KB (next 8-row group), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(128 >> 4) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46);
}

// kind::f16 instruction descriptor: D f32, A and B bf16, both K-major, N=64, M=64.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) | ((64u >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    const uint32_t zero = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate), "r"(zero)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t* v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

struct Smem {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint32_t tmem;
    int abort;
};

constexpr int kSmemHead = 1024;   // Smem, padded so that the tiles start 1 KB aligned
static_assert(sizeof(Smem) <= kSmemHead, "barrier block too large");

__global__ void __launch_bounds__(kBsrThreads, 2) bsr_kernel(const __grid_constant__ BsrArgs a) {
    extern __shared__ __align__(1024) unsigned char smem[];
    const int kStages = a.stages;
    Smem& S = *reinterpret_cast<Smem*>(smem);               // barriers first, then the tiles
    unsigned char* stA = smem + kSmemHead;                  // [stages][8 KB] weight tiles
    unsigned char* stB = stA + kStages * kTileBytes;        // [stages][8 KB] spike tiles
    volatile int* abort = &S.abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&S.tfull[i], 1);
            mbar_init(&S.tempty[i], 4);
        }
        mbar_init(&S.drain, 1);
        S.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        // two 64-column fp32 accumulators
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem)),
                     "r"(128u)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem;

    auto fail = [&]() {
        *abort = 1;
        if (a.err) atomicCAS(a.err, 0, ERR_BSR_TIMEOUT);
    };

    if (warp == 0) {
        // The warp reads 32 column indices per coalesced load; lane 0 issues
        // the copies (no dependent global load per block).
        long long it = 0;
        int stage = 0;          // it % stages
        uint32_t phase = 0;     // (it / stages) & 1
        bool ok = true;
        const uint64_t stream_once = policy_evict_first(), keep = policy_evict_last();
        for (int r = blockIdx.x; r < a.n_rows && ok; r += gridDim.x) {
            const int b0 = a.row_ptr[r], b1 = a.row_ptr[r + 1];
            for (int base = b0; base < b1 && ok; base += 32) {
                const int my_col = base + lane < b1 ? a.col_idx[base + lane] : 0;
                const int cnt = b1 - base < 32 ? b1 - base : 32;
                for (int q = 0; q < cnt; ++q, ++it) {
                    const int c = __shfl_sync(0xffffffffu, my_col, q);
                    bool got = true;
                    if (lane == 0) {
                        const int s = stage;
                        const uint32_t ph = phase;
                        if (++stage == kStages) {
                            stage = 0;
                            phase ^= 1u;
                        }
                        got = mbar_wait(&S.empty[s], ph ^ 1u, abort);
                        if (got) {
                            mbar_expect_tx(&S.full[s], 2 * kTileBytes);
                            bulk_load(stA + s * kTileBytes, a.tiles + static_cast<long long>(base + q) * kTileElems,
                                      kTileBytes, &S.full[s], stream_once);
                            bulk_load(stB + s * kTileBytes, a.spikes + static_cast<long long>(c) * kTileElems,
                                      kTileBytes, &S.full[s], keep);
                        } else {
                            fail();
                        }
                    }
                    if (!__shfl_sync(0xffffffffu, got, 0)) {
                        ok = false;
                        break;
                    }
                }
            }
        }
        // the copies still in flight land before the CTA exits
        if (lane == 0) {
            for (long long q = it - 1; q >= 0 && q >= it - kStages; --q)   // `it` counts issued stages
                mbar_wait(&S.full[q % kStages], static_cast<uint32_t>((q / kStages) & 1), nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            long long it = 0, rr = 0;
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int r = blockIdx.x; r < a.n_rows && ok; r += gridDim.x) {
                const int b0 = a.row_ptr[r], b1 = a.row_ptr[r + 1];
                if (b0 == b1) continue;
                const int acc = static_cast<int>(rr & 1);
                if (!mbar_wait(&S.tempty[acc], static_cast<uint32_t>(((rr >> 1) & 1) ^ 1), abort)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + static_cast<uint32_t>(acc * 64);
                for (int b = b0; b < b1; ++b, ++it) {
                    const int s = stage;
                    const uint32_t ph = phase;
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    if (!mbar_wait(&S.full[s], ph, abort)) {
                        fail();
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t pa = smem_u32(stA + s * kTileBytes), pb = smem_u32(stB + s * kTileBytes);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma(d, smem_desc(pa + kk * 256), smem_desc(pb + kk * 256), (b > b0 || kk > 0) ? 1u : 0u);
                    tc_commit(&S.empty[s]);
                }
                if (!ok) break;
                tc_commit(&S.tfull[acc]);
                ++rr;
            }
            // every MMA issued has completed before the accumulators are freed
            tc_commit(&S.drain);
            mbar_wait(&S.drain, 0, nullptr);
        }
    } else {
        const int sub = warp & 3;   // TMEM lanes 32*sub .. 32*sub+31 (M=64: rows 16*sub .. 16*sub+15)
        long long rr = 0;
        for (int r = blockIdx.x; r < a.n_rows; r += gridDim.x) {
            const int b0 = a.row_ptr[r], b1 = a.row_ptr[r + 1];
            if (b0 == b1) continue;
            const int acc = static_cast<int>(rr & 1);
            // every lane waits; the warp goes on only if all saw the phase complete
            const bool got = mbar_wait(&S.tfull[acc], static_cast<uint32_t>((rr >> 1) & 1), abort);
            if (!__all_sync(0xffffffffu, got)) {
                if (lane == 0) fail();
                break;
            }
            tc_fence_after();
            uint32_t v[64];
            const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * sub) << 16) + static_cast<uint32_t>(acc * 64);
            tc_ld32(taddr, v);
            tc_ld32(taddr + 32, v + 32);
            tc_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.tempty[acc]);
            if (lane < 16) {
                const long long post = static_cast<long long>(r) * 64 + 16 * sub + lane;
                float4* dst = reinterpret_cast<float4*>(a.i_syn + post * 64);
#pragma unroll
                for (int q = 0; q < 16; ++q) {
                    float4 x = dst[q];
                    x.x += __uint_as_float(v[4 * q + 0]);
                    x.y += __uint_as_float(v[4 * q + 1]);
                    x.z += __uint_as_float(v[4 * q + 2]);
                    x.w += __uint_as_float(v[4 * q + 3]);
                    dst[q] = x;
                }
            }
            ++rr;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(128u)
                                : "memory");
}

// Element (row, k) of a 64x64 tile in the K-major canonical order.
__host__ __device__ __forceinline__ int tile_off(int row, int k) {
    return (row >> 3) * 512 + (k >> 3) * 64 + (row & 7) * 8 + (k & 7);
}

// Row-major blocks [n][64 post][64 pre] -> tiles.
__global__ void pack_blocks_kernel(const uint16_t* blocks, long long n_blocks, uint16_t* tiles) {
    const long long total = n_blocks * kTileElems;
    for (long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long b = e / kTileElems;
        const int rem = static_cast<int>(e - b * kTileElems);
        tiles[b * kTileElems + tile_off(rem >> 6, rem & 63)] = blocks[e];
    }
}

__device__ __forceinline__ uint16_t bf16_bits(float x) {
    // 0 and 1 are exact in bf16: the upper half of the fp32 pattern
    return static_cast<uint16_t>(__float_as_uint(x) >> 16);
}

// Spikes [n_pre][64 trials] (0/1 floats) -> spike tiles (rows = trial, K = pre).
__global__ void pack_spikes_kernel(const float* s, int n_pre_blocks, uint16_t* tiles) {
    const long long total = static_cast<long long>(n_pre_blocks) * kTileElems;
    for (long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long pre = e >> 6;
        const int trial = static_cast<int>(e & 63);
        const long long c = pre >> 6;
        const float x = s[e];
        tiles[c * kTileElems + tile_off(trial, static_cast<int>(pre & 63))] = x != 0.0f ? bf16_bits(1.0f) : 0;
    }
}

__global__ void unpack_spikes_kernel(const uint16_t* tiles, int n_pre_blocks, float* s) {
    const long long total = static_cast<long long>(n_pre_blocks) * kTileElems;
    for (long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
         e += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long pre = e >> 6;
        const int trial = static_cast<int>(e & 63);
        const long long c = pre >> 6;
        const uint16_t v = tiles[c * kTileElems + tile_off(trial, static_cast<int>(pre & 63))];
        s[e] = __uint_as_float(static_cast<uint32_t>(v) << 16);
    }
}

// Bernoulli(p) spikes of step `step`, drawn per (pre neuron, group of four
// trials) from Philox keyed by (neuron, trial group, step): one thread per
// (pre block, 8-neuron K group, 4-trial group) writes 4 x 16 B.
__global__ void spikes_kernel(uint64_t seed, long long step, float p, int n_pre_blocks, uint16_t* tiles) {
    const long long total = static_cast<long long>(n_pre_blocks) * 8 * 16;
    for (long long u = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; u < total;
         u += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long c = u / 128;
        const int rem = static_cast<int>(u - c * 128);
        const int kg = rem >> 4, tg = rem & 15;
        uint32_t bits[4][8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t pre = static_cast<uint32_t>(c * 64 + kg * 8 + k);
            const U4 x = philox4x32_10(U4{pre, static_cast<uint32_t>(tg), static_cast<uint32_t>(step),
                                          kStreamBsr ^ static_cast<uint32_t>(step >> 32)},
                                       seed);
            bits[0][k] = u01(x.x) < p;
            bits[1][k] = u01(x.y) < p;
            bits[2][k] = u01(x.z) < p;
            bits[3][k] = u01(x.w) < p;
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int trial = tg * 4 + t;
            uint4 w;
            const uint32_t one = bf16_bits(1.0f);
            w.x = (bits[t][0] ? one : 0u) | ((bits[t][1] ? one : 0u) << 16);
            w.y = (bits[t][2] ? one : 0u) | ((bits[t][3] ? one : 0u) << 16);
            w.z = (bits[t][4] ? one : 0u) | ((bits[t][5] ? one : 0u) << 16);
            w.w = (bits[t][6] ? one : 0u) | ((bits[t][7] ? one : 0u) << 16);
            *reinterpret_cast<uint4*>(tiles + c * kTileElems + tile_off(trial, kg * 8)) = w;
        }
    }
}

int grid_for_elems(long long n) {
    const long long b = (n + 255) / 256;
    return static_cast<int>(std::max<long long>(1, std::min<long long>(b, 32LL * sm_count_current())));
}

}  // namespace
}  // namespace nrn

using namespace nrn;

extern "C" nrn_status_t nrn_cuda_bsr_pack(const uint16_t* blocks, int64_t n_blocks, uint16_t* tiles,
                                          nrn_stream_t stream) {
    NRN_CHECK_ARG(n_blocks >= 0, "nrn_cuda_bsr_pack: negative block count");
    if (n_blocks == 0) return NRN_OK;
    NRN_CHECK_ARG(blocks && tiles, "nrn_cuda_bsr_pack: null array");
    pack_blocks_kernel<<<grid_for_elems(n_blocks * kTileElems), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        blocks, n_blocks, tiles);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

extern "C" nrn_status_t nrn_cuda_bsr_pack_spikes(const float* spikes, int32_t n_pre_blocks, uint16_t* tiles,
                                                 nrn_stream_t stream) {
    NRN_CHECK_ARG(n_pre_blocks >= 0 && spikes && tiles, "nrn_cuda_bsr_pack_spikes: bad arguments");
    if (n_pre_blocks == 0) return NRN_OK;
    pack_spikes_kernel<<<grid_for_elems(static_cast<long long>(n_pre_blocks) * kTileElems), 256, 0,
                         reinterpret_cast<cudaStream_t>(stream)>>>(spikes, n_pre_blocks, tiles);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

extern "C" nrn_status_t nrn_cuda_bsr_unpack_spikes(const uint16_t* tiles, int32_t n_pre_blocks, float* spikes,
                                                   nrn_stream_t stream) {
    NRN_CHECK_ARG(n_pre_blocks >= 0 && spikes && tiles, "nrn_cuda_bsr_unpack_spikes: bad arguments");
    if (n_pre_blocks == 0) return NRN_OK;
    unpack_spikes_kernel<<<grid_for_elems(static_cast<long long>(n_pre_blocks) * kTileElems), 256, 0,
                           reinterpret_cast<cudaStream_t>(stream)>>>(tiles, n_pre_blocks, spikes);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

extern "C" nrn_status_t nrn_cuda_bsr_spikes(uint64_t seed, int64_t step, float p, int32_t n_pre_blocks,
                                            uint16_t* tiles, nrn_stream_t stream) {
    NRN_CHECK_ARG(n_pre_blocks >= 0 && tiles && p >= 0.0f && p <= 1.0f, "nrn_cuda_bsr_spikes: bad arguments");
    if (n_pre_blocks == 0) return NRN_OK;
    spikes_kernel<<<grid_for_elems(static_cast<long long>(n_pre_blocks) * 128), 256, 0,
                    reinterpret_cast<cudaStream_t>(stream)>>>(seed, step, p, n_pre_blocks, tiles);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

extern "C" nrn_status_t nrn_cuda_bsr_propagate(const nrn_bsr_t* w, const uint16_t* spike_tiles, float* i_syn,
                                               int32_t* err, nrn_stream_t stream) {
    NRN_CHECK_ARG(w != nullptr, "nrn_cuda_bsr_propagate: null weights");
    NRN_CHECK_ARG(w->n_post_blocks >= 0 && w->n_pre_blocks >= 0 && w->n_blocks >= 0,
                  "nrn_cuda_bsr_propagate: negative sizes");
    if (w->n_post_blocks == 0 || w->n_blocks == 0) return NRN_OK;
    NRN_CHECK_ARG(w->row_ptr && w->col_idx && w->tiles && spike_tiles && i_syn,
                  "nrn_cuda_bsr_propagate: null array");
    NRN_CHECK_ARG(w->n_blocks < (int64_t(1) << 31), "nrn_cuda_bsr_propagate: at most 2^31 - 1 blocks");
    for (const void* p : {static_cast<const void*>(w->tiles), static_cast<const void*>(spike_tiles),
                          static_cast<const void*>(i_syn)})
        NRN_CHECK_ARG(reinterpret_cast<uintptr_t>(p) % 16 == 0, "nrn_cuda_bsr_propagate: arrays must be 16-byte aligned");
    BsrArgs a;
    a.n_rows = w->n_post_blocks;
    a.row_ptr = w->row_ptr;
    a.col_idx = w->col_idx;
    a.tiles = w->tiles;
    a.spikes = spike_tiles;
    a.i_syn = i_syn;
    a.err = err;
    // Pipeline shape: CTAs per SM and stages per CTA (defaults measured on
    // B200; NRN_BSR_CTAS / NRN_BSR_STAGES override them for tuning).
    // Two CTAs per SM, 6 stages each (2 independent pipelines): 89% of the
    // measured HBM bandwidth at 262,144^2 neurons, against 46-61% for one.
    int ctas = 2, stages = 6;
    if (const char* v = std::getenv("NRN_BSR_CTAS")) ctas = std::max(1, std::min(2, std::atoi(v)));
    if (ctas == 1) stages = kMaxStages;
    if (const char* v = std::getenv("NRN_BSR_STAGES")) stages = std::max(2, std::min(kMaxStages, std::atoi(v)));
    if (ctas == 2 && stages > 6) stages = 6;   // two CTAs share one SM's shared memory
    a.stages = stages;
    const size_t smem = kSmemHead + 2 * static_cast<size_t>(stages) * kTileBytes;
    NRN_CUDA_TRY(cudaFuncSetAttribute(bsr_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    const int grid = std::min(a.n_rows, ctas * sm_count_current());
    bsr_kernel<<<grid, kBsrThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(a);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}
