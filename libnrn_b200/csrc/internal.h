// internal.h -- device-side building blocks shared by the engine.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "nrn_cuda.h"

namespace nrn {

// A projection's synapses on the device, sorted by (source, delay).
struct DevCsr {
    int32_t n_src = 0, n_tgt = 0;
    int32_t dmin = 1, nd = 1;
    int64_t nnz = 0;
    int64_t* seg_ptr = nullptr;   // [n_src*nd + 1]
    uint32_t* tgt = nullptr;      // [nnz]
    float* w = nullptr;           // [nnz]
    float* mod = nullptr;         // [nnz] or null
    int64_t* orig = nullptr;      // [nnz] index in the caller's list, or null
    int32_t max_seg = 0;          // longest (source, delay) segment
    int32_t max_row = 0;          // longest row (all delays of one source)
    int32_t max_in = 0;           // longest in-list
    // target-major index (plasticity)
    int64_t* in_ptr = nullptr;    // [n_tgt+1]
    uint32_t* in_syn = nullptr;   // [nnz]
    uint32_t* in_src = nullptr;   // [nnz]
};

void free_csr(DevCsr& c);

// Builds `c` from a synapse list in device memory (src < 0 entries are
// dropped).  keep_orig retains each synapse's index in the input list.
nrn_status_t build_csr(DevCsr& c, int32_t n_src, int32_t n_tgt, const int32_t* src, const int32_t* tgt,
                       const float* w, const uint8_t* delay, const float* mod, int64_t n_in, bool keep_orig,
                       cudaStream_t s);
// Adds the target-major index (in_ptr/in_syn/in_src).
nrn_status_t build_transpose(DevCsr& c, cudaStream_t s);

// Fixed in/out-degree generation into device arrays of length rows*degree;
// entries whose target falls outside [keep_lo, keep_hi) get src = -1.
struct GenArgs {
    int out_degree;
    int degree;
    uint32_t gen_id;
    int32_t n_src, src_offset;   // source population range (global ids)
    int32_t col_offset, col_n;   // candidate column range (global ids)
    int32_t row_offset, n_rows;  // rows: targets (in) or sources (out)
    int32_t keep_lo, keep_hi;    // kept target range (global ids)
    int32_t dmin, dmax;
    float w_lo, w_span;
    uint64_t seed;
};
nrn_status_t generate(const GenArgs& g, int32_t* src, int32_t* tgt, float* w, uint8_t* delay, cudaStream_t s);

int sm_count_current();

// Deferred-potentiation STDP (plastic.cu).
enum { PLASTIC_DELIVER = 0, PLASTIC_LTD = 1, PLASTIC_FLUSH = 2 };
struct PlasticArgs {
    int32_t n_src = 0, nd = 1, dmin = 1;
    const int64_t* seg_ptr = nullptr;
    const uint32_t* tgt = nullptr;
    float* w = nullptr;
    const float* mod = nullptr;
    float* acc = nullptr;
    const float* x_pre = nullptr;
    const float* x_post = nullptr;
    const float* spike_src = nullptr;
    const float* spike_tgt = nullptr;
    nrn_spike_hist_t hist_src{};
    float a_plus = 0, a_minus = 0, lr = 0, w_min = 0, w_max = 0, decay_pre = 1;
    int32_t* seg_last = nullptr;      // [n_src*nd] weights applied through this step
    float* seg_x = nullptr;           // [n_src*nd] x_pre at that step
    const float* x_snap = nullptr;    // [snap_depth][n_src]
    int32_t snap_period = 16, snap_depth = 64;
    const int4* post_recent = nullptr;
    const int32_t* post_ring = nullptr;
    const int32_t* post_cnt = nullptr;
    int32_t post_ring_k = 64;
    int64_t sweep_rows = 0;           // rows refreshed per step by the sweep
    int64_t sweep_period = 1;         // steps for the sweep to cover every row
    int* err = nullptr;
    unsigned long long* events = nullptr;
};
nrn_status_t plastic_rows(const PlasticArgs& a, int mode, long long step_off, const long long* step_base,
                          cudaStream_t s);

// The engine's spike raster buffers (for entry points outside engine.cu).
struct EngineRasterView {
    int device = 0;
    cudaStream_t stream = nullptr;
    int32_t* step = nullptr;
    int32_t* gid = nullptr;
    unsigned long long* count = nullptr;
    int64_t cap = 0;
    int64_t* flushed = nullptr;   // host counter of spikes already read
};
nrn_status_t engine_raster_view(nrn_engine* e, EngineRasterView* v);

// Sorts n raster entries in place by (step, global id).
nrn_status_t sort_raster(int32_t* step, int32_t* gid, int64_t n, cudaStream_t s);

}  // namespace nrn
