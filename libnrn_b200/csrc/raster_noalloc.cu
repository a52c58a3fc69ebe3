// raster_noalloc.cu -- reading the spike raster without allocating memory.
//
// nrn_engine_raster sorts the recorded spikes on the GPU with temporary
// device buffers that it allocates and frees on every call.  Some callers
// cannot do that: a host loop that drains the raster while the simulation
// keeps running in real time, or a process that has handed all free device
// memory to other work.  There, cudaMalloc/cudaFree can stall the device
// (cudaFree synchronises) or fail.  nrn_engine_raster_noalloc does the same
// work inside one fixed scratch array that lives in this library's device
// memory for as long as the library is loaded.
//
// Limits and sharing:
//   * at most kNoAllocMaxSpikes spikes per call (NRN_ERR_CAPACITY beyond,
//     leaving the raster untouched, so the caller can read it with
//     nrn_engine_raster instead);
//   * the scratch array (kNoAllocScratchBytes) exists once per GPU and is
//     shared by every engine on that GPU: two calls whose work overlaps on
//     the GPU (different threads, different engines) race on it;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress; make that first call before any stream capture.
#include <cuda_runtime.h>

#include <cub/device/device_radix_sort.cuh>
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace nrn {
namespace {

constexpr int64_t kNoAllocMaxSpikes = int64_t(1) << 17;      // 131,072 spikes per call
constexpr size_t kKeyBytes = static_cast<size_t>(kNoAllocMaxSpikes) * sizeof(unsigned long long);
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;    // 4 MiB: two key buffers + sort temp
constexpr int kMaxDevices = 64;

// One per GPU that loads the library; its contents persist between calls
// (nothing in it needs to start at zero: the sort overwrites what it uses).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {};
size_t g_sort_temp_bytes[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up on the
// first call for that device, with the device current).
nrn_status_t scratch_for_device(int dev, unsigned char** out, size_t* temp_bytes) {
    NRN_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "nrn_engine_raster_noalloc: device index too large");
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
        // The sort's temporary storage for the largest call must fit after
        // the two key buffers.
        size_t bytes = 0;
        cub::DoubleBuffer<unsigned long long> db(nullptr, nullptr);
        e = cub::DeviceRadixSort::SortKeys(nullptr, bytes, db, static_cast<int>(kNoAllocMaxSpikes), 0, 64);
        if (e != cudaSuccess) return cuda_fail(e, "radix sort size query");
        if (bytes > kNoAllocScratchBytes - 2 * kKeyBytes)
            return fail(NRN_ERR_CAPACITY, "nrn_engine_raster_noalloc: scratch array too small for the sort");
        g_sort_temp_bytes[dev] = bytes;
        g_scratch_addr[dev] = p;
    }
    *out = static_cast<unsigned char*>(g_scratch_addr[dev]);
    *temp_bytes = g_sort_temp_bytes[dev];
    return NRN_OK;
}

__global__ void pack_keys(const int32_t* step, const int32_t* gid, int64_t n, unsigned long long* key) {
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x)
        key[k] = (static_cast<unsigned long long>(static_cast<uint32_t>(step[k])) << 32) |
                 static_cast<uint32_t>(gid[k]);
}

__global__ void unpack_keys(const unsigned long long* key, int64_t n, int32_t* step, int32_t* gid) {
    for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        step[k] = static_cast<int32_t>(key[k] >> 32);
        gid[k] = static_cast<int32_t>(key[k] & 0xFFFFFFFFull);
    }
}

}  // namespace
}  // namespace nrn

extern "C" nrn_status_t nrn_engine_raster_noalloc(nrn_engine* e, int32_t* step, int32_t* gid, int64_t cap,
                                                  int64_t* n) {
    using namespace nrn;
    NRN_CHECK_ARG(e != nullptr && n != nullptr, "nrn_engine_raster_noalloc: null argument");
    EngineRasterView v;
    NRN_TRY(engine_raster_view(e, &v));
    NRN_CUDA_TRY(cudaSetDevice(v.device));
    unsigned long long cnt = 0;
    NRN_CUDA_TRY(cudaMemcpyAsync(&cnt, v.count, sizeof(cnt), cudaMemcpyDeviceToHost, v.stream));
    NRN_CUDA_TRY(cudaStreamSynchronize(v.stream));
    *n = static_cast<int64_t>(cnt);
    if (cnt == 0) return NRN_OK;
    if (static_cast<int64_t>(cnt) > v.cap)
        return fail(NRN_ERR_CAPACITY, "spike raster overflowed: read it more often");
    if (static_cast<int64_t>(cnt) > kNoAllocMaxSpikes)
        return fail(NRN_ERR_CAPACITY, "nrn_engine_raster_noalloc reads at most 131072 spikes per call (" +
                                          std::to_string(cnt) + " recorded); read more often or use nrn_engine_raster");
    NRN_CHECK_ARG(step != nullptr && gid != nullptr, "nrn_engine_raster_noalloc: null output");
    if (static_cast<int64_t>(cnt) > cap) return fail(NRN_ERR_CAPACITY, "output buffer too small for the raster");
    unsigned char* scratch = nullptr;
    size_t temp_bytes = 0;
    NRN_TRY(scratch_for_device(v.device, &scratch, &temp_bytes));
    auto* keys_a = reinterpret_cast<unsigned long long*>(scratch);
    auto* keys_b = reinterpret_cast<unsigned long long*>(scratch + kKeyBytes);
    void* temp = scratch + 2 * kKeyBytes;
    const int64_t m = static_cast<int64_t>(cnt);
    const int blocks = static_cast<int>((m + 255) / 256);
    pack_keys<<<blocks, 256, 0, v.stream>>>(v.step, v.gid, m, keys_a);
    NRN_CUDA_TRY(cudaGetLastError());
    cub::DoubleBuffer<unsigned long long> db(keys_a, keys_b);
    size_t bytes = temp_bytes;
    NRN_CUDA_TRY(cub::DeviceRadixSort::SortKeys(temp, bytes, db, static_cast<int>(m), 0, 64, v.stream));
    unpack_keys<<<blocks, 256, 0, v.stream>>>(db.Current(), m, v.step, v.gid);
    NRN_CUDA_TRY(cudaGetLastError());
    NRN_CUDA_TRY(cudaMemcpyAsync(step, v.step, m * sizeof(int32_t), cudaMemcpyDeviceToHost, v.stream));
    NRN_CUDA_TRY(cudaMemcpyAsync(gid, v.gid, m * sizeof(int32_t), cudaMemcpyDeviceToHost, v.stream));
    NRN_CUDA_TRY(cudaMemsetAsync(v.count, 0, sizeof(unsigned long long), v.stream));
    NRN_CUDA_TRY(cudaStreamSynchronize(v.stream));
    *v.flushed += m;
    return NRN_OK;
}
