// internal.h -- device-side building blocks shared by the engine.
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>

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
    // deterministic delivery: target-major index in CSR order (source, delay,
    // the caller's list order), with each synapse's source and delay
    int64_t* det_ptr = nullptr;   // [n_tgt+1]
    uint32_t* det_syn = nullptr;  // [nnz] CSR position
    uint32_t* det_src = nullptr;  // [nnz]
    uint8_t* det_delay = nullptr; // [nnz]
};

void free_csr(DevCsr& c);

// Builds `c` from a synapse list in device memory (src < 0 entries are
// dropped).  keep_orig retains each synapse's index in the input list.
nrn_status_t build_csr(DevCsr& c, int32_t n_src, int32_t n_tgt, const int32_t* src, const int32_t* tgt,
                       const float* w, const uint8_t* delay, const float* mod, int64_t n_in, bool keep_orig,
                       cudaStream_t s);
// Adds the target-major index (in_ptr/in_syn/in_src).
nrn_status_t build_transpose(DevCsr& c, cudaStream_t s);
// Adds the deterministic delivery index (det_*).
nrn_status_t build_det_index(DevCsr& c, cudaStream_t s);

// Deterministic delivery (deliver.cu): each target's input is the sum, in
// a fixed order (projection; source; delay; the caller's list order), of the
// weights of its synapses whose source spiked `delay` steps ago -- the
// order of a sequential CPU loop, so the result does not depend on thread
// timing.  Spikes are read from per-population flag rings
// ([ring][n_global] bytes, row s % ring = spiked at step s).
struct DetProj {
    const int64_t* ptr = nullptr;
    const uint32_t* syn = nullptr;
    const uint32_t* src = nullptr;
    const uint8_t* delay = nullptr;
    const float* w = nullptr;
    const float* mod = nullptr;
    const uint8_t* flags = nullptr;   // the source population's flag ring
    int64_t flag_n = 0;               // its row length (the population's size)
};
struct DetAcc {
    float* acc = nullptr;             // [n] written (not added)
    int32_t n = 0;
    int32_t nproj = 0;
    DetProj proj[8];
};
nrn_status_t det_deliver(const DetAcc& a, int32_t ring, long long step_off, const long long* step_base,
                         unsigned long long* events, cudaStream_t s);
// Row (step % ring) of a flag ring from a population's 0/1 spike vector.
nrn_status_t det_flags(const float* spike, int32_t n, uint8_t* flags, int32_t ring, long long step_off,
                       const long long* step_base, cudaStream_t s);

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

// Random (Erdos-Renyi) and distance-dependent connectivity (connect.cu).
struct RandArgs {
    int32_t rule = 0;                 // NRN_GEN_ER or NRN_GEN_DISTANCE
    uint64_t seed = 0;
    uint32_t gen_id = 0;
    int32_t n_src = 0;                // source population size
    int32_t n_tgt = 0;                // target population size
    int32_t tgt_lo = 0, n_rows = 0;   // this GPU's targets (population indices)
    int32_t tgt_gid_offset = 0;       // global id of target 0
    int32_t same_pop = 0;             // skip autapses
    double p = 0.0, log1mp = 0.0;     // ER: p and det_log(1 - p)
    double spacing_src = 0.0, spacing_tgt = 0.0, inv_two_sigma_sq = 0.0, p_min = 0.0;
    double half_window = -1.0;        // distance rule: window half width (< 0: all sources)
    int32_t dmin = 1, dmax = 1;
    float w_lo = 0.0f, w_span = 0.0f;
};
// A synapse list in device memory (source and target population indices,
// target relative to this GPU's first).
struct DevSynList {
    int64_t n = 0;
    int32_t* src = nullptr;
    int32_t* tgt = nullptr;
    float* w = nullptr;
    uint8_t* delay = nullptr;
    void release() {
        if (src) cudaFree(src);
        if (tgt) cudaFree(tgt);
        if (w) cudaFree(w);
        if (delay) cudaFree(delay);
        src = tgt = nullptr;
        w = nullptr;
        delay = nullptr;
        n = 0;
    }
};
nrn_status_t generate_random(const RandArgs& a, DevSynList* out, cudaStream_t s);

int sm_count_current();

// Neuron updates of several populations; populations of the same model and
// kind share one launch (neuron.cu).
nrn_status_t pop_step_group(const nrn_pop_step_t* list, int n, cudaStream_t s);

// This step's drive of several populations drawn ahead into out[q] (one
// launch for up to four populations; neuron.cu).
nrn_status_t drive_fill_group(const nrn_pop_step_t* list, float* const* out, int n, cudaStream_t s);

// Pair STDP applied by segment walks (plastic.cu).  Steps are int32.
enum { WALK_STEP = 0, WALK_FLUSH = 1 };
struct WalkArgs {
    int32_t n_src = 0, nd = 1, dmin = 1, max_seg = 0;
    const int64_t* seg_ptr = nullptr;
    const uint32_t* tgt = nullptr;
    float* w = nullptr;
    const float* mod = nullptr;
    float* acc = nullptr;
    nrn_spike_hist_t hist_src{};      // spike history of the (whole) source population
    int32_t* seg_last = nullptr;      // [n_src*nd] events applied through this step
    float* seg_x = nullptr;           // [n_src*nd] x_pre at that step
    // spike steps of the sources (index in the source population): newest
    // four in src_recent; older ones in src_ring/src_cnt for [src_lo, src_hi)
    const int4* src_recent = nullptr;
    const int32_t* src_ring = nullptr;
    const int32_t* src_cnt = nullptr;
    int32_t src_lo = 0, src_hi = 0;
    // spike steps of the targets (local index)
    const int4* tgt_recent = nullptr;
    const int32_t* tgt_ring = nullptr;
    const int32_t* tgt_cnt = nullptr;
    int32_t ring_k = 64;
    // source trace at window ends: x_j(m*win - 1) at (m % pre_depth) * n_src + j
    // (window-major: the window-end update is coalesced; a walk reads its
    // windows one lane each)
    const float* pre_snap = nullptr;
    int32_t pre_depth = 1;
    // target trace at every step: x(t) in row t % post_depth ([depth][n_tgt])
    const float* post_ring = nullptr;
    int32_t post_depth = 1;
    int32_t n_tgt = 0;
    int32_t win = 1;
    float decay_pre = 1, decay_post = 1, a_plus = 0, a_minus = 0, lr = 0, w_min = 0, w_max = 0;
    int64_t sweep_rows = 0;           // rows looked at per step by the sweep
    int32_t sweep_period = 1;         // steps for the sweep to pass every row
    int32_t stale = 1;                // the sweep walks a segment not walked for this many steps
    int* err = nullptr;
    unsigned long long* events = nullptr;
    // [3] unit counters of the launches (zero before a run's first launch)
    unsigned int* work_ctr = nullptr;
    int32_t no_deliver = 0;           // 1: update weights only (deterministic delivery)
};
nrn_status_t walk_launch(const WalkArgs& a, int mode, long long step_off, const long long* step_base,
                         cudaStream_t s);

// Window-end bookkeeping of one population (exchange.cu): trace snapshots
// from the window's spike masks, spike steps of the sources other ranks
// own, mask reset.
struct SnapTask {
    float* snap = nullptr;            // x_j(m*win - 1) at (m % depth) * (hi - lo) + (j - lo)
    int32_t depth = 1;
    int32_t lo = 0, hi = 0;           // population indices covered (snap column = j - lo)
    float decay = 1;
};
struct WindowArgs {
    int32_t n = 0;                    // population size (all ranks)
    uint32_t* mask = nullptr;         // [n] bit u: spiked at window step u
    SnapTask task[4];
    int32_t n_task = 0;
    int4* recent = nullptr;           // [n] or null; updated outside [own_lo, own_hi)
    int32_t own_lo = 0, own_hi = 0;
    const int32_t* seg_last = nullptr;   // segments of a walk projection from this population
    int32_t seg_nd = 0;
    int32_t win = 1;
    int* err = nullptr;
};
nrn_status_t window_launch(const WindowArgs& a, long long step_off, const long long* step_base, cudaStream_t s);

// Spike exchange: unpacks the gathered per-rank window buffers of one
// population into its spike history ring (and the masks of the spikes of
// other ranks).
struct UnpackArgs {
    const int32_t* recv = nullptr;    // rank r's block at recv + r * rank_stride
    int64_t rank_stride = 0;
    int64_t pop_off = 0;              // this population's block offset inside a rank block
    int32_t cap = 0;                  // id capacity of a block (after win counts and the total)
    int32_t world = 1, rank = 0;
    int32_t win = 1;
    nrn_spike_hist_t hist{};
    uint32_t* mask = nullptr;         // or null
    int* err = nullptr;
};
nrn_status_t unpack_launch(const UnpackArgs& a, long long step_off, const long long* step_base, cudaStream_t s);

// The engine's NCCL communicator (comm.cu): blocking (its collectives are
// captured in CUDA graphs), every host wait on it bounded by timeout_s; on
// an error or a timeout the communicator is aborted (*c becomes null) and
// NRN_ERR_COMM returned.
nrn_status_t comm_init(ncclComm_t* out, int world, const uint8_t id[128], int rank, double timeout_s);
// After an NCCL call that returned r.
nrn_status_t comm_settle(ncclComm_t* c, ncclResult_t r, double timeout_s, const char* what);
// Waits for stream s of a partitioned engine; *stuck is set when the stream
// did not drain even after the abort.
nrn_status_t comm_wait_stream(ncclComm_t* c, cudaStream_t s, double timeout_s, bool* stuck);
nrn_status_t comm_abort(ncclComm_t* c);
nrn_status_t comm_destroy(ncclComm_t* c, double timeout_s);

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
// Device buffers of the raster sort, kept between reads (grown on demand).
struct RasterSortScratch {
    unsigned long long* a = nullptr;
    unsigned long long* b = nullptr;
    void* tmp = nullptr;
    size_t tmp_bytes = 0;
    int64_t cap = 0;
    void release() {
        if (a) cudaFree(a);
        if (b) cudaFree(b);
        if (tmp) cudaFree(tmp);
        a = b = nullptr;
        tmp = nullptr;
        tmp_bytes = 0;
        cap = 0;
    }
};
// Sorts n raster entries by (step, gid) in place on stream s; gid < 2^gid_bits,
// step < 2^step_bits (the sort reads only those key bits).
nrn_status_t sort_raster(int32_t* step, int32_t* gid, int64_t n, int gid_bits, int step_bits, RasterSortScratch& sc,
                         cudaStream_t s);

}  // namespace nrn
