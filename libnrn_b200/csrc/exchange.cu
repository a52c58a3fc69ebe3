// exchange.cu -- window-end work: gathered spikes into the history rings,
// STDP trace snapshots.
//
// A network partitioned over GPUs by neuron index steps in windows of `win`
// steps, win <= the smallest synaptic delay: a spike emitted in one window
// arrives in a later one, so each GPU only needs the other GPUs' spikes
// once per window.  During a window, each population's update appends the
// ids of its spiking neurons (index in the whole population) to a send
// buffer, [win counts][total][ids, window step by window step].  At the window's
// end the per-rank buffers are gathered (one all-gather over NCCL,
// engine.cu) and unpacked here into the population's spike history ring:
// step s in slot s % depth, the ranks' ids one after the other.
//
// The window end is also when the STDP trace snapshots are taken: for every
// neuron whose spikes some plastic projection needs, the trace value at the
// window's last step is the previous snapshot advanced through the window,
//     x <- x*decay + (spiked at u ? 1 : 0),   u = 0 .. win-1,
// with the spikes read from the window's bit mask (one bit per step) -- the
// same operations, in the same order, as the reference's per-step decay and
// increment of its traces (src/plasticity/stdp.cpp:118-128).
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace nrn {
namespace {

constexpr int kThreads = 256;
enum { ERR_ORDER = 3, ERR_EXCHANGE = 4 };

__global__ void __launch_bounds__(kThreads) window_kernel(const __grid_constant__ WindowArgs a, long long step_off,
                                                          const long long* step_base) {
    const long long step = step_off + (step_base ? *step_base : 0);   // last step of the window
    const int ws = static_cast<int>(step + 1 - a.win);
    const int m = static_cast<int>((step + 1) / a.win);               // snapshot written now
    for (long long j = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; j < a.n;
         j += static_cast<long long>(gridDim.x) * blockDim.x) {
        const uint32_t bits = a.mask[j];
        for (int k = 0; k < a.n_task; ++k) {
            const SnapTask& t = a.task[k];
            if (j < t.lo || j >= t.hi) continue;
            // window-major rows: consecutive neurons are adjacent (coalesced)
            const long long col = j - t.lo, cols = t.hi - t.lo;
            float x = t.snap[static_cast<long long>((m - 1) & (t.depth - 1)) * cols + col];
            for (int u = 0; u < a.win; ++u) x = x * t.decay + (((bits >> u) & 1u) ? 1.0f : 0.0f);
            t.snap[static_cast<long long>(m & (t.depth - 1)) * cols + col] = x;
        }
        if (bits == 0) continue;
        a.mask[j] = 0;
        if (a.recent != nullptr && (j < a.own_lo || j >= a.own_hi)) {
            // spikes of another rank's neuron: shift them in, oldest first
            int4 r = a.recent[j];
            int first = -1;
            for (int u = 0; u < a.win; ++u) {
                if (!((bits >> u) & 1u)) continue;
                if (first < 0) first = ws + u;
                r = make_int4(ws + u, r.x, r.y, r.z);
            }
            a.recent[j] = r;
            // A segment of this source already walked past that spike (only
            // possible when it spikes twice within one delay) applied its
            // updates without it.
            if (a.seg_last != nullptr)
                for (int k = 0; k < a.seg_nd; ++k)
                    if (a.seg_last[j * a.seg_nd + k] >= first) atomicCAS(a.err, 0, ERR_ORDER);
        }
    }
}

// One block per (rank, window step): copies that rank's ids of that step
// into the step's history slot after those of the lower ranks.
__global__ void __launch_bounds__(kThreads) unpack_kernel(const __grid_constant__ UnpackArgs a, long long step_off,
                                                          const long long* step_base) {
    const long long step = step_off + (step_base ? *step_base : 0);   // last step of the window
    const long long ws = step + 1 - a.win;
    const int r = blockIdx.x / a.win;
    const int u = blockIdx.x % a.win;
    const int32_t* blk = a.recv + r * a.rank_stride + a.pop_off;
    int before = 0;   // this rank's ids of earlier window steps
    for (int q = 0; q < u; ++q) before += blk[q];
    int n = blk[u];
    int off = 0;      // ids of lower ranks at this step
    int total = 0;
    for (int q = 0; q < a.world; ++q) {
        const int c = a.recv[q * a.rank_stride + a.pop_off + u];
        if (q < r) off += c;
        total += c;
    }
    if (before + n > a.cap || off + n > a.hist.cap) {
        if (threadIdx.x == 0) atomicCAS(a.err, 0, ERR_EXCHANGE);
        const int room = a.cap - before < a.hist.cap - off ? a.cap - before : a.hist.cap - off;
        n = room > 0 ? room : 0;
    }
    const int slot = static_cast<int>((ws + u) % a.hist.depth);
    const int32_t* src = blk + a.win + 1 + before;   // [win counts | total | ids]
    int32_t* dst = a.hist.ids + static_cast<long long>(slot) * a.hist.cap + off;
    const bool other = r != a.rank && a.mask != nullptr;
    for (int q = threadIdx.x; q < n; q += blockDim.x) {
        const int id = src[q];
        dst[q] = id;
        if (other) atomicOr(a.mask + id, 1u << u);
    }
    if (r == 0 && threadIdx.x == 0) a.hist.count[slot] = total < a.hist.cap ? total : a.hist.cap;
}

}  // namespace

nrn_status_t window_launch(const WindowArgs& a, long long step_off, const long long* step_base, cudaStream_t s) {
    NRN_CHECK_ARG(a.win >= 1 && a.win <= 32 && a.n_task >= 0 && a.n_task <= 4, "window: bad arguments");
    for (int k = 0; k < a.n_task; ++k)
        NRN_CHECK_ARG(a.task[k].depth > 0 && (a.task[k].depth & (a.task[k].depth - 1)) == 0,
                      "window: snapshot depth must be a power of two");
    if (a.n <= 0) return NRN_OK;
    const int blocks = static_cast<int>(std::min<long long>((a.n + kThreads - 1) / kThreads, 16LL * sm_count_current()));
    window_kernel<<<blocks, kThreads, 0, s>>>(a, step_off, step_base);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

nrn_status_t unpack_launch(const UnpackArgs& a, long long step_off, const long long* step_base, cudaStream_t s) {
    NRN_CHECK_ARG(a.world >= 1 && a.win >= 1 && a.win <= 32, "unpack: bad arguments");
    unpack_kernel<<<a.world * a.win, kThreads, 0, s>>>(a, step_off, step_base);
    NRN_CUDA_TRY(cudaGetLastError());
    return NRN_OK;
}

}  // namespace nrn
