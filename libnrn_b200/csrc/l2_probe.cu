// l2_probe.cu -- throughput of random memory operations on this GPU: float
// reductions, 16- and 4-byte loads at random addresses of L2-resident
// arrays, shared-memory reductions, and random 64-byte chunks against a
// sequential read of a 4 GiB array.  These are the operations spike
// delivery and the STDP walks are made of; their rates bound those kernels.
// Every index is masked into its power-of-two sized buffer.
//
//   l2_probe      (built by libnrn_b200/build.py into libnrn_b200/_lib/)
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>

#define CK(x) do { cudaError_t e = (x); if (e != cudaSuccess) { printf("%s: %s\n", #x, cudaGetErrorString(e)); return 1; } } while (0)

__device__ __forceinline__ uint32_t hash(uint32_t x) {
    x ^= x >> 16; x *= 0x7feb352dU; x ^= x >> 15; x *= 0x846ca68bU; x ^= x >> 16; return x;
}

__global__ void red_rand(float* acc, uint32_t mask, long long n_ev) {
    long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long nt = (long long)gridDim.x * blockDim.x;
    for (long long k = tid; k < n_ev; k += nt) atomicAdd(acc + (hash((uint32_t)k) & mask), 1.0f);
}

__global__ void ld16_rand(const int4* tab, uint32_t mask, long long n_ev, int* out) {
    long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long nt = (long long)gridDim.x * blockDim.x;
    int s = 0;
    for (long long k = tid; k < n_ev; k += nt) { int4 v = tab[hash((uint32_t)k) & mask]; s += v.x ^ v.w; }
    if (s == 0x12345) out[0] = s;
}

__global__ void ld4_rand(const float* tab, uint32_t mask, long long n_ev, float* out) {
    long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long nt = (long long)gridDim.x * blockDim.x;
    float s = 0;
    for (long long k = tid; k < n_ev; k += nt) s += tab[hash((uint32_t)k) & mask];
    if (s == 123.25f) out[0] = s;
}

// dependent-free: 4 independent loads per iteration
__global__ void ld4_rand_ilp(const float* tab, uint32_t mask, long long n_ev, float* out) {
    long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long nt = (long long)gridDim.x * blockDim.x;
    float s = 0;
    for (long long k = tid; k + 3 * nt < n_ev; k += 4 * nt) {
        float a = tab[hash((uint32_t)k) & mask], b = tab[hash((uint32_t)(k + nt)) & mask];
        float c = tab[hash((uint32_t)(k + 2 * nt)) & mask], d = tab[hash((uint32_t)(k + 3 * nt)) & mask];
        s += a + b + c + d;
    }
    if (s == 123.25f) out[0] = s;
}

__global__ void smem_red(long long n_ev_per_block, float* out) {
    __shared__ float acc[8192];
    for (int i = threadIdx.x; i < 8192; i += blockDim.x) acc[i] = 0;
    __syncthreads();
    for (long long k = threadIdx.x; k < n_ev_per_block; k += blockDim.x)
        atomicAdd(acc + (hash((uint32_t)(k + blockIdx.x * 7777)) & 8191), 1.0f);
    __syncthreads();
    if (threadIdx.x == 0) out[blockIdx.x] = acc[0];
}

// random 64-byte chunks of a big array (DRAM), 4 lanes x 16 B per chunk
__global__ void dram_rand64(const int4* big, uint64_t mask_chunks, long long n_chunks, int* out) {
    long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long nt = (long long)gridDim.x * blockDim.x;
    int s = 0;
    for (long long k = tid; k < 4 * n_chunks; k += nt) {
        uint64_t c = ((uint64_t)hash((uint32_t)(k >> 2)) * 2654435761ull) & mask_chunks;
        int4 v = big[c * 4 + (k & 3)];
        s += v.x ^ v.y;
    }
    if (s == 0x12345) out[0] = s;
}

// streaming copy-like read (DRAM seq)
__global__ void dram_seq(const int4* big, long long n, int* out) {
    long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long nt = (long long)gridDim.x * blockDim.x;
    int s = 0;
    for (long long k = tid; k < n; k += nt) { int4 v = big[k]; s += v.x ^ v.y; }
    if (s == 0x12345) out[0] = s;
}

// The STDP walk's memory pattern per plastic event: at one random target i,
// a 16-byte load (its newest spike steps), a 4-byte load (its trace) and a
// float reduction (its input); with `stream`, also the synapse's sequential
// target index and weight read and the weight written back (12 B).
__global__ void walk_like(const int4* recent, const float* trace, float* acc, uint32_t mask, long long n_ev,
                          const uint32_t* tgt, float* w, int stream, float* out) {
    long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long nt = (long long)gridDim.x * blockDim.x;
    float s = 0;
    for (long long k = tid; k < n_ev; k += nt) {
        const uint32_t i = (stream ? tgt[k] : hash((uint32_t)k)) & mask;
        const int4 r = recent[i];
        const float x = trace[i];
        const float wv = stream ? w[k] : 1.0f;
        const float w1 = wv + (r.x == 0x7fffffff ? 1.0f : 0.0f) * x;
        if (stream) w[k] = w1;
        atomicAdd(acc + i, w1);
        s += x;
    }
    if (s == 123.25f) out[0] = s;
}

// Static delivery per event: a float reduction at a random target, with the
// synapse's sequential target index and weight (8 B).
__global__ void deliver_like(float* acc, uint32_t mask, long long n_ev, const uint32_t* tgt, const float* w) {
    long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long nt = (long long)gridDim.x * blockDim.x;
    for (long long k = tid; k < n_ev; k += nt) atomicAdd(acc + (tgt[k] & mask), w[k]);
}

__global__ void fill_hash(uint32_t* t, long long n) {
    long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long nt = (long long)gridDim.x * blockDim.x;
    for (long long k = tid; k < n; k += nt) t[k] = hash((uint32_t)k * 2654435761u + 17u);
}

int main() {
    int sms = 0; cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    float* acc; int4* tab16; float* tab4; int* outi; float* outf; int4* big;
    const uint32_t N1 = 1u << 20;   // 1M floats = 4 MB
    const uint32_t N16 = 1u << 20;  // 1M int4 = 16 MB
    const size_t BIG = size_t(1) << 32;  // 4 GiB
    CK(cudaMalloc(&acc, N1 * 4)); CK(cudaMalloc(&tab16, N16 * 16)); CK(cudaMalloc(&tab4, N1 * 4));
    CK(cudaMalloc(&outi, 4096 * 4)); CK(cudaMalloc(&outf, 8192 * 4)); CK(cudaMalloc(&big, BIG));
    CK(cudaMemset(acc, 0, N1 * 4)); CK(cudaMemset(tab16, 1, N16 * 16)); CK(cudaMemset(tab4, 0, N1 * 4));
    CK(cudaMemset(big, 1, BIG));
    cudaEvent_t a, b; cudaEventCreate(&a); cudaEventCreate(&b);
    const long long EV = 1ll << 26;
    for (int bps : {4, 8}) {
        int grid = sms * bps;
        float ms;
        for (int rep = 0; rep < 2; ++rep) {
            cudaEventRecord(a); red_rand<<<grid, 256>>>(acc, N1 - 1, EV); cudaEventRecord(b); CK(cudaEventSynchronize(b));
            cudaEventElapsedTime(&ms, a, b);
        }
        printf("blocks/SM %d  RED.F32 random 4MB: %.1f G/s\n", bps, EV / (ms * 1e6));
        for (int rep = 0; rep < 2; ++rep) {
            cudaEventRecord(a); ld16_rand<<<grid, 256>>>(tab16, N16 - 1, EV, outi); cudaEventRecord(b); CK(cudaEventSynchronize(b));
            cudaEventElapsedTime(&ms, a, b);
        }
        printf("blocks/SM %d  LD.128 random 16MB: %.1f G/s\n", bps, EV / (ms * 1e6));
        for (int rep = 0; rep < 2; ++rep) {
            cudaEventRecord(a); ld4_rand<<<grid, 256>>>(tab4, N1 - 1, EV, outf); cudaEventRecord(b); CK(cudaEventSynchronize(b));
            cudaEventElapsedTime(&ms, a, b);
        }
        printf("blocks/SM %d  LD.32 random 4MB: %.1f G/s\n", bps, EV / (ms * 1e6));
        for (int rep = 0; rep < 2; ++rep) {
            cudaEventRecord(a); ld4_rand_ilp<<<grid, 256>>>(tab4, N1 - 1, EV, outf); cudaEventRecord(b); CK(cudaEventSynchronize(b));
            cudaEventElapsedTime(&ms, a, b);
        }
        printf("blocks/SM %d  LD.32 random 4MB ilp4: %.1f G/s\n", bps, EV / (ms * 1e6));
        const long long per_block = EV / grid;
        for (int rep = 0; rep < 2; ++rep) {
            cudaEventRecord(a); smem_red<<<grid, 256>>>(per_block, outf); cudaEventRecord(b); CK(cudaEventSynchronize(b));
            cudaEventElapsedTime(&ms, a, b);
        }
        printf("blocks/SM %d  shared RED random: %.1f G/s\n", bps, per_block * grid / (ms * 1e6));
        const long long NCH = 1ll << 24;   // 16M chunks of 64 B
        for (int rep = 0; rep < 2; ++rep) {
            cudaEventRecord(a); dram_rand64<<<grid, 256>>>(big, (BIG / 64) - 1, NCH, outi); cudaEventRecord(b); CK(cudaEventSynchronize(b));
            cudaEventElapsedTime(&ms, a, b);
        }
        printf("blocks/SM %d  DRAM random 64B chunks (4GB): %.1f G chunks/s = %.0f GB/s\n", bps, NCH / (ms * 1e6), NCH * 64 / (ms * 1e6));
        for (int rep = 0; rep < 2; ++rep) {
            cudaEventRecord(a); dram_seq<<<grid, 256>>>(big, BIG / 16, outi); cudaEventRecord(b); CK(cudaEventSynchronize(b));
            cudaEventElapsedTime(&ms, a, b);
        }
        printf("blocks/SM %d  DRAM seq read 4GB: %.0f GB/s\n", bps, BIG / (ms * 1e6));
    }
    {
        // mixed patterns at the walk's array sizes (1M targets), 8 blocks/SM
        const long long E2 = 1ll << 26;
        uint32_t* tg; float* wv;
        CK(cudaMalloc(&tg, E2 * 4)); CK(cudaMalloc(&wv, E2 * 4));
        fill_hash<<<sms * 8, 256>>>(tg, E2);
        CK(cudaMemset(wv, 0, E2 * 4));
        const int grid = sms * 8;
        float ms;
        for (int st = 0; st < 2; ++st) {
            for (int rep = 0; rep < 2; ++rep) {
                cudaEventRecord(a);
                walk_like<<<grid, 256>>>(tab16, tab4, acc, N1 - 1, E2, tg, wv, st, outf);
                cudaEventRecord(b); CK(cudaEventSynchronize(b));
                cudaEventElapsedTime(&ms, a, b);
            }
            printf("walk-like event (LD.128 + LD.32 + RED at one random target%s): %.1f G events/s = %.1f G random ops/s\n",
                   st ? ", + 12 B sequential synapse stream" : "", E2 / (ms * 1e6), 3.0 * E2 / (ms * 1e6));
        }
        for (int rep = 0; rep < 2; ++rep) {
            cudaEventRecord(a); deliver_like<<<grid, 256>>>(acc, N1 - 1, E2, tg, wv); cudaEventRecord(b);
            CK(cudaEventSynchronize(b));
            cudaEventElapsedTime(&ms, a, b);
        }
        printf("delivery-like event (RED at a random target + 8 B sequential synapse stream): %.1f G events/s\n",
               E2 / (ms * 1e6));
        cudaFree(tg); cudaFree(wv);
    }
    CK(cudaGetLastError());
    return 0;
}
