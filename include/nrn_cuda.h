/*
 * nrn_cuda.h -- C ABI of libnrn_b200's device layer (libnrn_cuda.so).
 *
 * The B200 engine for libnrn's per-timestep simulation hot path.  Plain C:
 * raw device pointers, sizes, plain structs and CUDA streams; no C++ or
 * LibTorch types cross this boundary.  Every entry point returns an
 * nrn_status_t; nrn_last_error() gives the message of the last failure on
 * the calling thread.
 *
 * Two levels:
 *
 *  1. Kernel entry points (stateless, enqueue on the given stream):
 *       nrn_cuda_pop_step     one fused neuron update of a population
 *                             (replaces the reference's internal
 *                             nrn::neuron::cuda::{lif,adex,izhikevich}_forward_cuda,
 *                             declared in src/neuron/lif.cpp:7-21,
 *                             src/neuron/adex.cpp:7-28,
 *                             src/neuron/izhikevich.cpp:7-19)
 *       nrn_cuda_deliver      event-driven spike delivery through a
 *                             source-major CSR (replaces the per-block
 *                             torch::mv loop of connection_deliver,
 *                             src/connectivity/connect.cpp:36-79, and the stub
 *                             launch_synaptic_current_block_dense,
 *                             src/synapse/kernels/synapse_kernels.cu:56-79)
 *       nrn_cuda_stdp_*       pair STDP (src/plasticity/stdp.cpp:43-141)
 *       nrn_cuda_bsr_propagate batched-trial block-sparse product on the
 *                             tensor cores (the stub's intended block-dense
 *                             matmul, synapse_kernels.cu:30-51, for many trials)
 *
 *  2. Engine entry points (a network resident on one GPU, stepped in CUDA
 *     graphs), which the C++ nrn:: layer's sim_create/sim_step/sim_run
 *     (src/simulation/runner.cpp:17-173) drive:
 *       nrn_engine_create / _add_population / _add_projection /
 *       _set_stdp / _finalize / _run / _sync / _raster / _weights / _destroy
 *
 * Spike semantics follow the reference's sim_step: a spike emitted at step s
 * through a synapse of delay d is added to the target's input at step s + d,
 * before the target's update of that step (SpikeBuffer::read(d),
 * src/simulation/spike_buffer.cpp:32-49).
 */
#ifndef NRN_CUDA_H
#define NRN_CUDA_H

#include <stdint.h>

#if defined(__GNUC__)
#define NRN_API __attribute__((visibility("default")))
#else
#define NRN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* A CUDA stream (cudaStream_t); NULL is the legacy default stream. */
typedef struct CUstream_st* nrn_stream_t;

typedef enum {
    NRN_OK = 0,
    NRN_ERR_INVALID = 1,      /* bad argument (reference: TORCH_CHECK failure) */
    NRN_ERR_CUDA = 2,         /* CUDA runtime error                             */
    NRN_ERR_OOM = 3,          /* device allocation failed                       */
    NRN_ERR_CAPACITY = 4,     /* a fixed-capacity buffer overflowed             */
    NRN_ERR_UNSUPPORTED = 5,  /* no device / wrong architecture                 */
    NRN_ERR_COMM = 6,         /* collective (NCCL) failure                      */
    NRN_ERR_TIMEOUT = 7,      /* a bounded device-side wait gave up             */
    NRN_ERR_STATE = 8         /* call out of order (e.g. run before finalize)   */
} nrn_status_t;

NRN_API const char* nrn_status_string(nrn_status_t s);
NRN_API const char* nrn_last_error(void);
/* Library version "major.minor.patch" and the compiled device architecture. */
NRN_API const char* nrn_version(void);

/* ------------------------------------------------------------------------ */
/* Neuron models                                                            */
/* ------------------------------------------------------------------------ */

enum { NRN_MODEL_LIF = 0, NRN_MODEL_ADEX = 1, NRN_MODEL_IZH = 2 };

/* Parameter slots (param[] / uniform[] below), in the reference's option
 * order (include/nrn/neuron/options.h):
 *   LIF : 0 v_rest 1 v_thresh 2 v_reset 3 tau_m 4 tau_ref 5 c_m 6 i_bg
 *   AdEx: 0 v_rest 1 v_thresh 2 v_reset 3 v_peak 4 tau_m 5 tau_w 6 tau_ref
 *         7 c_m 8 g_l 9 a 10 b 11 delta_t 12 i_bg
 *   Izh : 0 a 1 b 2 c 3 d 4 v_peak                                          */
#define NRN_MAX_PARAMS 13

/* External drive drawn on the device per (neuron, step) from Philox4x32-10
 * keyed by (seed; global id, step, 0, 0x44524956). */
enum {
    NRN_DRIVE_NONE = 0,
    NRN_DRIVE_POISSON_CURRENT = 1,   /* i_syn += amp * Poisson(lambda)          */
    NRN_DRIVE_GAUSS_CURRENT = 2,     /* i_syn += mean + std * N(0,1)            */
    NRN_DRIVE_POISSON_GEXC = 3       /* gin_exc += amp * Poisson(lambda)        */
};

typedef struct {
    int32_t kind;
    float p0;            /* lambda per step (Poisson) or mean (Gauss)        */
    float p1;            /* amplitude (Poisson) or standard deviation        */
    uint64_t seed;
} nrn_drive_t;

/* One update of a population: reads the input, integrates one step, writes
 * the spike flags and appends the ids of spiking neurons.  Operation order
 * and rounding follow the reference's CPU path (each operation rounded to
 * fp32, no fused multiply-add), so LIF and Izhikevich agree bit for bit and
 * AdEx to the last-bit difference of exp. */
typedef struct {
    int32_t model;
    int32_t n;
    int32_t gid_offset;        /* global id of neuron 0 (drive counter)     */
    int32_t pad0;
    double dt;                 /* seconds; 0 performs the initialising update */
    float* v;                  /* [n] membrane potential                    */
    float* aux;                /* [n] w (AdEx) / u (Izh); NULL for LIF      */
    float* refractory;         /* [n] remaining refractory time; NULL (Izh) */
    float* spike;              /* [n] 0/1 output, or NULL                   */
    float* i_syn;              /* [n] input current, read then zeroed; NULL = 0 */
    /* conductance input (AdEx only; all NULL for current-based input) */
    float* g_exc;              /* [n] conductance state                      */
    float* g_inh;
    float* gin_exc;            /* [n] conductance input this step, read then zeroed */
    float* gin_inh;
    float tau_syn_exc, tau_syn_inh, e_exc, e_inh;
    const float* param[NRN_MAX_PARAMS];   /* per-neuron arrays, or NULL      */
    float uniform[NRN_MAX_PARAMS];        /* used where param[k] is NULL     */
    nrn_drive_t drive;
    int64_t step;              /* absolute step index (drive counter)       */
    const int64_t* step_base;  /* if non-NULL, the step is *step_base + step */
    int32_t* spike_ids;        /* compacted local ids of spiking neurons, or NULL */
    int32_t* spike_count;      /* [1] incremented by the number appended    */
    /* When hist_depth > 0, spike_ids/spike_count are the bases of a spike
     * history ring (nrn_spike_hist_t): the ids go to slot step % hist_depth,
     * i.e. spike_ids + slot * hist_cap and spike_count + slot. */
    int32_t hist_depth;
    int32_t hist_cap;
    /* spike raster (the reference's spike recorder, src/monitor/spike_recorder.cpp):
     * if raster_gid is non-NULL every spike is also appended as (step, global id);
     * entries past raster_cap are counted but not written. */
    int32_t* raster_step;
    int32_t* raster_gid;
    unsigned long long* raster_count;
    int64_t raster_cap;
    /* Plasticity traces of this population, x <- x * decay + spike, updated
     * in the same pass at slow-clock steps (step % trace_slow_ratio == 0). */
    int32_t n_traces;          /* 0..NRN_MAX_TRACES                          */
    int32_t trace_slow_ratio;
    float* trace[4];
    float trace_decay[4];
    /* A trace slot k with trace_ring[k] non-NULL keeps every step's value:
     * x(t) in row t % trace_ring_depth of trace_ring[k] [depth][n], read
     * back from row (t-1) % depth (trace[k] is then unused). */
    float* trace_ring[4];
    int32_t trace_ring_depth;
    int32_t pad1;
    /* Spike-time history (for plasticity applied by segment walks): on a
     * spike at step t, post_recent[i] (int4:
     * latest four spike steps, newest first) shifts in t and t is appended
     * to post_ring[i*post_ring_k + post_cnt[i] % post_ring_k]. */
    int32_t* post_recent;      /* [n][4] or NULL                            */
    int32_t* post_ring;        /* [n][post_ring_k]                          */
    int32_t* post_cnt;         /* [n]                                       */
    int32_t post_ring_k;
    /* Spike exchange between the GPUs a network is partitioned over
     * (population split by neuron index).  id_offset is added to every
     * compacted id, so that ids index the whole population.  win > 0 marks
     * windows of win steps (win <= 32), window u = step % win:
     *   win_mask[i] |= 1 << u for each spike (window trace snapshots);
     *   with send_hdr non-NULL, the ids go to the window send buffer instead
     *   of the history ring: send_hdr[u] counts the ids of window step u,
     *   which follow those of steps 0..u-1 in send_ids[0 .. send_cap), and
     *   send_hdr[win] counts them all; overflow sets *err to 4. */
    int32_t id_offset;
    int32_t win;
    uint32_t* win_mask;        /* [n] or NULL                               */
    int32_t* send_hdr;         /* [win + 1] or NULL                         */
    int32_t* send_ids;         /* [send_cap]                                */
    int32_t send_cap;
    int32_t pad2;
    int32_t* err;              /* device error flag, or NULL                */
    /* Drive values of this step computed ahead (nrn_cuda_drive_fill with the
     * same arguments): if non-NULL, drive_values[i] replaces drawing the
     * drive of neuron i here -- the same numbers. */
    const float* drive_values;
    /* Per-neuron spike statistics updated at each spike, or NULL. */
    struct nrn_spike_stat* spike_stats;
    /* Synapse channels (nrn_syn_desc_t kinds), applied before the model
     * update: chan_in[c] is the input delivered this step (read, then
     * zeroed), chan_s[c] the decay state, chan_r[c] the rise state (DEXP,
     * AMPA).  n_chan = 0: none. */
    int32_t n_chan;
    int32_t chan_kind[4];
    float chan_e_rev[4];
    double chan_tau_rise[4], chan_tau_decay[4];
    float* chan_in[4];
    float* chan_s[4];
    float* chan_r[4];
} nrn_pop_step_t;

#define NRN_MAX_TRACES 4

NRN_API nrn_status_t nrn_cuda_pop_step(const nrn_pop_step_t* a, nrn_stream_t stream);
/* The external drive of the step described by a (drive, gid_offset, step,
 * step_base) into out[0..n): the values nrn_cuda_pop_step would draw, so
 * that they can be drawn ahead, concurrently with other work. */
NRN_API nrn_status_t nrn_cuda_drive_fill(const nrn_pop_step_t* a, float* out, nrn_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Spike delivery                                                           */
/* ------------------------------------------------------------------------ */

/* Spike statistics of one neuron, accumulated on the device at each of its
 * spikes (population statistics without reading the raster: rate = count /
 * time, CV of the inter-spike interval = sqrt(isi_sum2/m - (isi_sum/m)^2)
 * / (isi_sum/m) with m = count - 1 intervals).  No counterpart in the
 * reference, whose design notes list mean rate and CV_ISI as population
 * statistics to record. */
typedef struct nrn_spike_stat {
    int32_t last;              /* step of the last spike + 1 (0: none yet)  */
    int32_t count;             /* spikes                                    */
    int64_t isi_sum;           /* sum of the inter-spike intervals, steps   */
    int64_t isi_sum2;          /* sum of their squares                      */
} nrn_spike_stat_t;

/* Compacted spike history of one population: ring of depth `depth` steps,
 * slot s % depth holding the local ids of the neurons that spiked at s. */
typedef struct {
    int32_t* ids;              /* [depth][cap]                              */
    int32_t* count;            /* [depth]                                   */
    int32_t cap;
    int32_t depth;
} nrn_spike_hist_t;

/* A projection on the device: synapses sorted by (source, delay); the
 * synapses of source j with delay dmin + k are [seg_ptr[j*nd+k], seg_ptr[j*nd+k+1]). */
typedef struct {
    int32_t n_src;
    int32_t n_tgt;
    int32_t dmin;              /* smallest delay, steps (>= 1)              */
    int32_t nd;                /* number of delay values dmin .. dmin+nd-1  */
    int32_t src_hist;          /* index of the source's nrn_spike_hist_t    */
    int32_t max_seg;           /* longest (source, delay) segment           */
    const int64_t* seg_ptr;    /* [n_src*nd + 1]                            */
    const uint32_t* tgt;       /* [nnz] local target index                  */
    const float* w;            /* [nnz] weight                              */
    const float* mod;          /* [nnz] modulatory gain, or NULL (all 1)    */
    float* acc;                /* [n_tgt] target input accumulator          */
} nrn_proj_t;

#define NRN_MAX_PROJ 32
#define NRN_MAX_POPS 32

/* Delivers, for every projection, the spikes emitted at step - d through the
 * synapses of delay d, adding w (times mod) into acc.  Also clears the
 * history slot of `step` for every population (ready for this step's
 * updates).  step = *step_base + step_off when step_base is non-NULL. */
NRN_API nrn_status_t nrn_cuda_deliver(const nrn_proj_t* projs, int32_t nproj,
                              const nrn_spike_hist_t* hists, int32_t nhist,
                              int64_t step_off, const int64_t* step_base,
                              nrn_stream_t stream);
/* As nrn_cuda_deliver; also adds the number of synaptic events delivered to
 * *events (device counter) when it is non-NULL. */
NRN_API nrn_status_t nrn_cuda_deliver_counted(const nrn_proj_t* projs, int32_t nproj,
                                      const nrn_spike_hist_t* hists, int32_t nhist,
                                      int64_t step_off, const int64_t* step_base,
                                      unsigned long long* events, nrn_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Pair STDP (src/plasticity/stdp.cpp:43-141), per-neuron traces            */
/* ------------------------------------------------------------------------ */

typedef struct {
    nrn_proj_t proj;           /* the plastic projection (w is updated)     */
    float* w_mut;              /* == proj.w, writable                       */
    const int64_t* in_ptr;     /* [n_tgt+1] target-major index              */
    const uint32_t* in_syn;    /* [nnz] synapse position of each in-synapse */
    const uint32_t* in_src;    /* [nnz] its source                          */
    int32_t max_in;            /* longest in-list (max in-degree)           */
    int32_t max_row;           /* longest out-row (all delays of a source)  */
    float* x_pre;              /* [n_src] presynaptic trace                 */
    float* x_post;             /* [n_tgt] postsynaptic trace                */
    const float* spike_src;    /* [n_src] this step's 0/1 spikes            */
    const float* spike_tgt;    /* [n_tgt]                                   */
    nrn_spike_hist_t hist_src;
    nrn_spike_hist_t hist_tgt;
    float decay_pre, decay_post;      /* (float)exp(-dt/tau_plus|minus)     */
    float a_plus, a_minus;            /* a_minus as |A-|                    */
    float lr, w_min, w_max;
    int32_t slow_ratio;        /* update only when step % slow_ratio == 0   */
    int32_t traces_updated;    /* 1: the neuron updates already advanced x_pre/x_post */
} nrn_stdp_t;

/* Trace decay and increment, then the weight update of every synapse whose
 * source or target spiked at `step`, clamped to [w_min, w_max]. */
NRN_API nrn_status_t nrn_cuda_stdp_step(const nrn_stdp_t* s, int64_t step_off,
                                 const int64_t* step_base, nrn_stream_t stream);
/* Clamp all n weights to [lo, hi] (the reference clamps every entry on each
 * update; after one full clamp only changed weights can leave the range). */
NRN_API nrn_status_t nrn_cuda_clamp(float* w, int64_t n, float lo, float hi, nrn_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Block-dense connectivity (the nrn:: API's ConnectivityTensor layout)     */
/* ------------------------------------------------------------------------ */

/* Dense B x B blocks, CSR over target block rows; all arrays on the device,
 * float [n_blocks][B][B] for weights and masks.  Replaces the reference's
 * stub block-dense launcher (src/synapse/kernels/synapse_kernels.cu:56-79). */
typedef struct {
    const int32_t* row_ptr;          /* [n_target_blocks + 1] */
    const int32_t* col_idx;          /* [n_blocks]            */
    const float* weights;
    const float* structural_mask;
    const float* modulatory_mask;
    int64_t block_size;
    int64_t n_blocks;
    int64_t n_source;
    int64_t n_target;
} nrn_block_csr_t;

/* i_syn[t] += sum over the blocks of t's row of ((W*Ms)*Mm)[t,:] . spikes
 * (connection_deliver, src/connectivity/connect.cpp:36-79). */
NRN_API nrn_status_t nrn_cuda_block_deliver(const nrn_block_csr_t* c, const float* spikes, float* i_syn,
                                            nrn_stream_t stream);
/* One STDP update on block-dense weights with per-synapse traces
 * (stdp_update, src/plasticity/stdp.cpp:43-141).  params = {decay_pre,
 * decay_post, a_plus, |a_minus|, learning_rate, w_min, w_max}. */
NRN_API nrn_status_t nrn_cuda_block_stdp(const nrn_block_csr_t* c, float* weights, float* trace_pre,
                                         float* trace_post, const float* pre_spikes, const float* post_spikes,
                                         const float* params, nrn_stream_t stream);
/* Ids of the non-zero entries of x appended to ids (order within the
 * result unspecified); *count incremented. */
NRN_API nrn_status_t nrn_cuda_compact(const float* x, int64_t n, int32_t* ids, int32_t* count,
                                      nrn_stream_t stream);
/* out[i] = ring[(write_pos - delays[i]) mod depth][i]  (SpikeBuffer::read_batch). */
NRN_API nrn_status_t nrn_cuda_gather_ring(const float* ring, int64_t n, int64_t depth, int64_t write_pos,
                                          const int64_t* delays, float* out, nrn_stream_t stream);
/* dst[pos[k]] = src[k]. */
NRN_API nrn_status_t nrn_cuda_scatter(const float* src, const int64_t* pos, int64_t n, float* dst,
                                      nrn_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Batched block-sparse propagation (tensor cores)                          */
/* ------------------------------------------------------------------------ */

/* Block-sparse weights of 64x64 bf16 blocks, block-row CSR.  Each block is
 * stored as one 4096-element tile in the tensor core's K-major canonical
 * order (nrn_cuda_bsr_pack makes it from row-major [post][pre] blocks). */
typedef struct {
    int32_t n_post_blocks;     /* block rows: post neurons / 64             */
    int32_t n_pre_blocks;      /* block columns: pre neurons / 64           */
    int64_t n_blocks;
    const int32_t* row_ptr;    /* [n_post_blocks + 1]                       */
    const int32_t* col_idx;    /* [n_blocks]                                */
    const uint16_t* tiles;     /* [n_blocks][4096] bf16, 16-byte aligned    */
} nrn_bsr_t;

/* I[post][trial] += sum over blocks (r,c): W[r,c] . S[pre in c][trial], for
 * 64 trials at once: bf16 x bf16 products accumulated in fp32 (tcgen05).
 * i_syn is [n_post_blocks*64][64] fp32; spike_tiles holds one tile per pre
 * block (nrn_cuda_bsr_spikes / nrn_cuda_bsr_pack_spikes).  Replaces the
 * reference's block-dense kernel, launch_synaptic_current_block_dense
 * (src/synapse/kernels/synapse_kernels.cu:30-79, a stub there), for the
 * batched-trial case.  A device-side wait that times out sets *err to 5. */
NRN_API nrn_status_t nrn_cuda_bsr_propagate(const nrn_bsr_t* w, const uint16_t* spike_tiles, float* i_syn,
                                            int32_t* err, nrn_stream_t stream);
/* Row-major bf16 blocks [n_blocks][64 post][64 pre] -> tiles. */
NRN_API nrn_status_t nrn_cuda_bsr_pack(const uint16_t* blocks, int64_t n_blocks, uint16_t* tiles,
                                       nrn_stream_t stream);
/* 0/1 spikes [n_pre_blocks*64][64 trials] (float) <-> spike tiles. */
NRN_API nrn_status_t nrn_cuda_bsr_pack_spikes(const float* spikes, int32_t n_pre_blocks, uint16_t* tiles,
                                              nrn_stream_t stream);
NRN_API nrn_status_t nrn_cuda_bsr_unpack_spikes(const uint16_t* tiles, int32_t n_pre_blocks, float* spikes,
                                                nrn_stream_t stream);
/* Bernoulli(p) spikes of step `step` for 64 trials, Philox keyed by (pre
 * neuron, trial group, step) -- the same spikes for any launch shape. */
NRN_API nrn_status_t nrn_cuda_bsr_spikes(uint64_t seed, int64_t step, float p, int32_t n_pre_blocks,
                                         uint16_t* tiles, nrn_stream_t stream);

/* ------------------------------------------------------------------------ */
/* Engine: a network resident on one GPU                                   */
/* ------------------------------------------------------------------------ */

typedef struct nrn_engine nrn_engine;

typedef struct {
    int32_t model;
    int32_t n;                 /* neurons on this GPU                        */
    int32_t gid_offset;        /* global id of the population's neuron 0    */
    int32_t record;            /* 1: keep every spike in the raster          */
    /* Partitioned network (nrn_engine_set_partition): this GPU holds neurons
     * [local_offset, local_offset + n) of a population of n_global neurons.
     * 0, 0: the whole population (n_global = n). */
    int32_t n_global;
    int32_t local_offset;
    /* state of this GPU's neurons, caller-owned device arrays (the
     * reference's state tensors) */
    float* v;
    float* aux;
    float* refractory;
    float* spike;
    float* i_syn;
    /* conductance input: tau_syn_exc > 0 enables it (AdEx) */
    float tau_syn_exc, tau_syn_inh, e_exc, e_inh;
    const float* param[NRN_MAX_PARAMS];
    float uniform[NRN_MAX_PARAMS];
    nrn_drive_t drive;
} nrn_pop_desc_t;

/* Receptor of a projection: the target's input current, its AdEx
 * conductance inputs, or NRN_RECV_CHANNEL + c for synapse channel c of the
 * target population (nrn_engine_add_synapse_channel). */
enum { NRN_RECV_CURRENT = 0, NRN_RECV_GEXC = 1, NRN_RECV_GINH = 2, NRN_RECV_CHANNEL = 16 };

/* A synapse channel: per-neuron synapse state of a population, fused into
 * its neuron update.  These are the reference's synapse models, declared in
 * include/nrn/synapse/exponential.h:16-21, double_exponential.h:17-25 and
 * ampa.h:17-29 (their forward is a stub there,
 * src/synapse/exponential.cpp:37-42).  Each step, before the neuron
 * integrates, with `in` the weights delivered into the channel this step and
 * dec = (float)exp(-dt/tau):
 *   NRN_SYN_EXP : s = s*dec_decay + in;  I += s
 *   NRN_SYN_DEXP: s = s*dec_decay + in;  r = r*dec_rise + in;  I += s - r
 *   NRN_SYN_AMPA: s, r as DEXP; g = s - r;  I += g*(e_rev - v)
 * (AMPA's declared I_syn = g*(V - E_rev) is the outward membrane current;
 * the neuron models add inward current, hence e_rev - v). */
enum { NRN_SYN_EXP = 1, NRN_SYN_DEXP = 2, NRN_SYN_AMPA = 3 };
#define NRN_MAX_CHANNELS 4
typedef struct {
    int32_t kind;
    int32_t pad;
    double tau_rise;           /* s (DEXP, AMPA)                             */
    double tau_decay;          /* s                                          */
    double e_rev;              /* reversal potential (AMPA), the population's units */
} nrn_syn_desc_t;

/* Synapse list of a projection (host or device memory, see `on_device`),
 * any order; delays in steps.  The engine keeps its own copy. */
typedef struct {
    int32_t src_pop;
    int32_t tgt_pop;
    int32_t receptor;
    int32_t on_device;         /* 1: the arrays below are device pointers   */
    int64_t nnz;
    const int32_t* src;        /* [nnz] source index in the whole population */
    const int32_t* tgt;        /* [nnz] target index on this GPU            */
    const float* w;            /* [nnz]                                     */
    const uint8_t* delay;      /* [nnz] steps, >= 1                         */
    const float* mod;          /* [nnz] modulatory gain, or NULL            */
} nrn_proj_desc_t;

/* Connectivity generated on the device from Philox counters, so every GPU
 * of a partition and the host oracle draw the same synapses:
 *   NRN_GEN_FIXED    fixed in-degree (out_degree 0) or out-degree (1);
 *   NRN_GEN_ER       every (source, target) pair with probability p, the
 *                    rule of the reference's random topology
 *                    (src/connectivity/topology/random.cpp:25-95);
 *   NRN_GEN_DISTANCE pairs with probability max(exp(-d^2/(2 sigma^2)),
 *                    min_probability), d the distance of 1D positions
 *                    i * max_distance / n, the rule of the reference's
 *                    distance-dependent topology
 *                    (src/connectivity/topology/distance_dependent.cpp:28-144).
 * The reference draws these with the torch generator into block-dense
 * tensors (the nrn:: connect() path keeps that sequence); these draw per
 * synapse on the device, without the N_src x N_tgt storage. */
enum { NRN_GEN_FIXED = 0, NRN_GEN_ER = 1, NRN_GEN_DISTANCE = 2 };
typedef struct {
    int32_t src_pop;
    int32_t tgt_pop;
    int32_t receptor;
    int32_t out_degree;        /* 0: rows are targets, 1: rows are sources  */
    int32_t degree;
    int32_t gen_id;
    int32_t col_offset;        /* global id range the draws pick from       */
    int32_t col_n;
    int32_t dmin, dmax;
    float w_lo, w_span;
    uint64_t seed;
    int32_t rule;              /* NRN_GEN_*                                  */
    int32_t pad;
    double p;                  /* ER probability                             */
    double sigma, max_distance, min_probability;   /* distance rule          */
} nrn_gen_desc_t;

NRN_API nrn_status_t nrn_engine_create(nrn_engine** out, int device, double dt, int32_t slow_ratio);
NRN_API nrn_status_t nrn_engine_destroy(nrn_engine* e);
/* Multi-GPU: the network is partitioned by neuron index over `world` GPUs,
 * one engine (and process or thread) per GPU, each built with the same
 * calls on its slice of every population.  Spikes are exchanged with one
 * NCCL all-gather per window of min(smallest delay, 32) steps; `id` is an
 * NCCL unique id from nrn_comm_unique_id on one rank, passed to all (the
 * call blocks until every rank has made it).  max_rate_hz bounds the mean
 * firing rate of a population over a window (exchange buffer size); above
 * it the run fails with NRN_ERR_CAPACITY.  Call before adding populations.
 * Every rank must run the same step counts.  No counterpart in the
 * reference (its runner is single-device, src/simulation/runner.cpp). */
NRN_API nrn_status_t nrn_comm_unique_id(uint8_t id[128]);
/* Every host wait on the communicator is bounded (nrn_engine_set_comm_timeout,
 * default 120 s): its set-up here (on a helper thread), the layout
 * check in nrn_engine_finalize (every rank must build the same network:
 * otherwise NRN_ERR_COMM), and every wait on the engine stream of a
 * partitioned run (nrn_engine_sync, raster and weight reads, checkpoints).
 * A rank that stopped, ran other step counts or failed makes the others'
 * waits end with NRN_ERR_COMM: the communicator is aborted (its waiting
 * NCCL kernels end) and later runs return NRN_ERR_STATE. */
NRN_API nrn_status_t nrn_engine_set_partition(nrn_engine* e, int32_t rank, int32_t world, const uint8_t id[128],
                                              double max_rate_hz);
/* Time limit of the host waits on a partitioned engine (set before
 * nrn_engine_set_partition to bound its set-up too). */
NRN_API nrn_status_t nrn_engine_set_comm_timeout(nrn_engine* e, double seconds);
/* The bounded wait the engine uses: calls poll(ctx) until it returns > 0
 * (NRN_OK) or < 0 (NRN_ERR_COMM), spinning at first and then sleeping
 * between calls; NRN_ERR_TIMEOUT after timeout_s seconds.  Host only. */
NRN_API nrn_status_t nrn_comm_bounded_wait(int (*poll)(void*), void* ctx, double timeout_s);
/* Test hook: the next query of a communicator's asynchronous state reports
 * nccl_result (an ncclResult_t) instead of NCCL's own; 0 clears it.  Lets a
 * test drive the abort path with an error code, without a failing GPU. */
NRN_API nrn_status_t nrn_comm_fake_async_error(int32_t nccl_result);
NRN_API nrn_status_t nrn_engine_add_population(nrn_engine* e, const nrn_pop_desc_t* d, int32_t* id);
/* Update the uniform/per-neuron parameters of a population (between runs). */
NRN_API nrn_status_t nrn_engine_set_params(nrn_engine* e, int32_t pop, const float* const* param,
                                   const float* uniform);
NRN_API nrn_status_t nrn_engine_add_projection(nrn_engine* e, const nrn_proj_desc_t* d, int32_t* id);
/* Adds synapse channel *channel (0..NRN_MAX_CHANNELS-1) to population pop;
 * projections deliver into it with receptor NRN_RECV_CHANNEL + channel.
 * Before nrn_engine_finalize. */
NRN_API nrn_status_t nrn_engine_add_synapse_channel(nrn_engine* e, int32_t pop, const nrn_syn_desc_t* d,
                                                    int32_t* channel);
NRN_API nrn_status_t nrn_engine_generate_projection(nrn_engine* e, const nrn_gen_desc_t* g, int32_t* id,
                                            int64_t* nnz);
/* stdp = {tau_plus, tau_minus, a_plus, a_minus, w_min, w_max, learning_rate} */
NRN_API nrn_status_t nrn_engine_set_stdp(nrn_engine* e, int32_t proj, const double* stdp);
/* Deterministic delivery (before nrn_engine_finalize; one GPU): each
 * neuron input is the sum, in a fixed order -- projection by projection in
 * index order, each by source, then delay, then the order its synapses were
 * given -- of the weights
 * of the synapses whose source spiked `delay` steps ago: the order of a
 * sequential CPU loop, so results do not depend on thread timing and a
 * checkpointed run resumes bit for bit.  It visits every in-synapse of every
 * neuron each step (a test and reproducibility mode, not the fast path). */
NRN_API nrn_status_t nrn_engine_set_deterministic(nrn_engine* e, int32_t on);
/* Allocates the history and traces and runs the initialising update
 * (dt = 0, as sim_create does, src/simulation/runner.cpp:36-38). */
NRN_API nrn_status_t nrn_engine_finalize(nrn_engine* e, int32_t init_update);
/* Enqueues `steps` steps (CUDA graphs of `chunk` steps; 0 picks a size). */
NRN_API nrn_status_t nrn_engine_run(nrn_engine* e, int64_t steps, int32_t chunk);
/* Captures (without running them) the CUDA graphs that nrn_engine_run(e,
 * steps, chunk) would replay when started at step first_step, so that a
 * later run -- a timed one, or the first steps of a simulation -- captures
 * none. */
NRN_API nrn_status_t nrn_engine_prepare(nrn_engine* e, int64_t first_step, int64_t steps, int32_t chunk);
NRN_API nrn_status_t nrn_engine_sync(nrn_engine* e);
/* Sets the number of the next step (drive counters, slow-clock boundaries,
 * raster step numbers); spikes already in flight keep their ring slots. */
NRN_API nrn_status_t nrn_engine_set_step(nrn_engine* e, int64_t step);
NRN_API nrn_status_t nrn_engine_stream(nrn_engine* e, nrn_stream_t* stream);
NRN_API int64_t nrn_engine_step(const nrn_engine* e);
/* What a caller needs to pace its reads: the window (steps between spike
 * exchanges and trace snapshots; runs that start and end on window
 * boundaries replay the fewest distinct graphs), and the raster's capacity
 * in spikes over the neurons it records (a caller that reads the raster at
 * least every raster_capacity / recorded_neurons steps cannot overflow it).
 * Valid after nrn_engine_finalize. */
typedef struct {
    int32_t window;
    int32_t n_pops;
    int64_t raster_capacity;
    int64_t recorded_neurons;
    int64_t step;
} nrn_engine_info_t;
NRN_API nrn_status_t nrn_engine_info(const nrn_engine* e, nrn_engine_info_t* out);
/* Recorded spikes since the last call (host buffers), sorted by step and,
 * within a step, by ascending global id; *n receives the count
 * (if above cap, nothing is copied and NRN_ERR_CAPACITY is returned). */
NRN_API nrn_status_t nrn_engine_raster(nrn_engine* e, int32_t* step, int32_t* gid, int64_t cap, int64_t* n);
/* As nrn_engine_raster, but allocates no device memory, for callers that
 * cannot call cudaMalloc/cudaFree (a real-time loop draining spikes while
 * the simulation runs: allocation and free can stall the device; a process
 * whose device memory is spoken for).  No counterpart in the reference.
 * The sort runs in one fixed 4 MiB scratch array inside the library, one
 * per GPU, kept until the library is unloaded and shared by all engines on
 * that GPU: calls that overlap on the GPU race.  At most 131,072 spikes per
 * call; beyond that NRN_ERR_CAPACITY is returned and the raster is left for
 * nrn_engine_raster.  The first call on a device sets up the scratch
 * address (cudaGetSymbolAddress) and should come before any stream capture. */
NRN_API nrn_status_t nrn_engine_raster_noalloc(nrn_engine* e, int32_t* step, int32_t* gid, int64_t cap,
                                               int64_t* n);
/* State probes (the reference's state recorder, src/monitor/state_recorder.cpp:41-58,
 * which clones the state to the host at every recorded step): after every
 * step's neuron update, variable `var` (NRN_VAR_*) of this GPU's neurons of
 * population `pop` is copied into row (step % depth) of `ring`, a caller's
 * device array [depth][n], inside the engine's step graphs.  The caller
 * reads the rows at most depth steps later.  Adding or clearing probes
 * recaptures the graphs. */
enum { NRN_VAR_V = 0, NRN_VAR_AUX = 1, NRN_VAR_REFRACTORY = 2, NRN_VAR_SPIKE = 3, NRN_VAR_ISYN = 4 };
NRN_API nrn_status_t nrn_engine_add_probe(nrn_engine* e, int32_t pop, int32_t var, float* ring, int32_t depth,
                                          int32_t* id);
NRN_API nrn_status_t nrn_engine_clear_probes(nrn_engine* e);
/* Weights of a projection in the order the synapses were given, into a
 * device array of nnz floats (enqueued on the engine stream). */
NRN_API nrn_status_t nrn_engine_weights_device(nrn_engine* e, int32_t proj, float* out, int64_t n);
/* Current state pointers of a population (the caller re-allocated them). */
NRN_API nrn_status_t nrn_engine_set_state(nrn_engine* e, int32_t pop, float* v, float* aux, float* refractory,
                                          float* spike, float* i_syn);
/* Weights of a projection in the order the synapses were given (host). */
NRN_API nrn_status_t nrn_engine_weights(nrn_engine* e, int32_t proj, float* out, int64_t n);
NRN_API nrn_status_t nrn_engine_nnz(nrn_engine* e, int32_t proj, int64_t* nnz);
/* Runs `steps` steps without graphs, timing each phase with CUDA events on
 * the engine stream: ms[0] delivery, ms[1] neuron updates, ms[2] plasticity
 * (summed over the steps).  For profiling; results equal nrn_engine_run. */
NRN_API nrn_status_t nrn_engine_profile(nrn_engine* e, int64_t steps, double* ms);
/* Runs `steps` steps with every kernel on the engine stream one after the
 * other (no overlap), timing each with CUDA events: ms[0] external drive,
 * ms[1] static delivery, ms[2] STDP walks (plastic delivery), ms[3] neuron
 * updates, ms[4] per-step STDP kernels, ms[5] window ends (spike exchange,
 * trace snapshots), summed over the steps.  counts[0] events delivered by
 * the static delivery, counts[1] by the walks, counts[2] window ends,
 * counts[3] steps.  Results equal nrn_engine_run's. */
NRN_API nrn_status_t nrn_engine_profile_kernels(nrn_engine* e, int64_t steps, double* ms, int64_t* counts);
/* Counters: total spikes and delivered synaptic events since creation. */
NRN_API nrn_status_t nrn_engine_counters(nrn_engine* e, int64_t* spikes, int64_t* events);

/* Checkpoint of the engine's device state: neuron state and synaptic input,
 * spike histories, weights, plasticity state (traces, walk state, trace
 * snapshots and rings), step counter, event counter and the raster not yet
 * read.  Fills the reference's I/O stub (src/simulation/runner.cpp:222,
 * "save() -- stub, not yet implemented").  A checkpoint restores into an
 * engine built from the same network (same populations, projections and
 * partition), finalized; the run then continues as the saved one would.
 * A partitioned engine is checkpointed at window boundaries only (the
 * spike exchange holds nothing then); NRN_ERR_STATE otherwise.
 * nrn_engine_checkpoint_size gives the bytes of a checkpoint now; save
 * writes exactly that many into host memory; load reads them back and
 * returns NRN_ERR_INVALID for a checkpoint of another network. */
/* Spike statistics: enabled before nrn_engine_finalize (one
 * nrn_spike_stat_t per neuron of every population, zeroed), copied out for
 * this rank's neurons of a population (n = its local size), zeroed again by
 * reset.  They are part of a checkpoint. */
NRN_API nrn_status_t nrn_engine_enable_spike_stats(nrn_engine* e);
NRN_API nrn_status_t nrn_engine_spike_stats(nrn_engine* e, int32_t pop, nrn_spike_stat_t* out, int64_t n);
NRN_API nrn_status_t nrn_engine_spike_stats_reset(nrn_engine* e);
NRN_API nrn_status_t nrn_engine_checkpoint_size(nrn_engine* e, int64_t* bytes);
NRN_API nrn_status_t nrn_engine_checkpoint_save(nrn_engine* e, void* buf, int64_t bytes);
NRN_API nrn_status_t nrn_engine_checkpoint_load(nrn_engine* e, const void* buf, int64_t bytes);

#ifdef __cplusplus
}
#endif
#endif /* NRN_CUDA_H */
