/*
 * oracle_common.h -- shared definitions of the CPU oracle.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (libnrn_b200/) includes,
 * links or executes this file; only tests/, the smoke check and bench.py's
 * CPU-baseline leg use the oracle, as the checker.
 *
 * Contents:
 *   1. The network description shared by the C restatement (nrn_oracle.c)
 *      and the reference driver (ref_harness.cpp).  Both are filled from the
 *      same Python-side description through ctypes.
 *   2. Philox4x32-10 counter RNG (Salmon, Moraes, Dror, Shaw: "Parallel
 *      random numbers: as easy as 1, 2, 3", SC'11) and the samplers built on
 *      it (uniform, Poisson by inversion, normal by Box-Muller with a log
 *      and a cosine written from their series).  Every sampler uses only
 *      IEEE-754 binary32 +,-,*,/ and sqrt, each rounded separately, so the
 *      CUDA build (compiled with -fmad=false) draws bit-identical values.
 *   3. Per-neuron fp32 update steps that restate the reference CPU paths in
 *      their exact operation order (each torch op rounds to fp32):
 *        LIF         src/neuron/lif.cpp:80-97
 *        AdEx        src/neuron/adex.cpp:97-124
 *        Izhikevich  src/neuron/izhikevich.cpp:76-98
 *      Scalars that the reference passes as C++ doubles into float tensor
 *      ops (dt, 0.04, 5.0, 140.0, 0.5*dt_ms ...) are rounded to float first,
 *      as ATen does for a wrapped double scalar meeting a float tensor.
 *
 * The file must be compiled with -ffp-contract=off so that no a*b+c is fused.
 */
#ifndef NRN_ORACLE_COMMON_H
#define NRN_ORACLE_COMMON_H

#include <stdint.h>
#include <math.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* 1. Network description                                                    */
/* ------------------------------------------------------------------------ */

enum { ORC_LIF = 0, ORC_ADEX = 1, ORC_IZH = 2 };

/* Drive kinds: external input generated per (neuron, step) from Philox. */
enum {
    ORC_DRIVE_NONE = 0,
    ORC_DRIVE_POISSON_CURRENT = 1,   /* I += amp * Poisson(lambda)            */
    ORC_DRIVE_GAUSS_CURRENT = 2,     /* I += mean + std * N(0,1)              */
    ORC_DRIVE_POISSON_GEXC = 3       /* g_exc input += amp * Poisson(lambda)  */
};

/* Receptor a projection delivers into; ORC_RECV_CHANNEL + c: synapse
 * channel c of the target population (below). */
enum { ORC_RECV_CURRENT = 0, ORC_RECV_GEXC = 1, ORC_RECV_GINH = 2, ORC_RECV_CHANNEL = 16 };

/* Synapse channels: per-target synapse state of the reference's declared
 * synapse models (include/nrn/synapse/exponential.h:16-21,
 * double_exponential.h:17-25, ampa.h:17-29; their forward is a stub in the
 * reference, so these equations are restated from the declarations alone:
 * parity unpinned).  Each step, before the neuron integrates, with `in` the
 * weights delivered into the channel this step:
 *   EXP : s = s*dec_decay + in;               I += s
 *   DEXP: s = s*dec_decay + in; r = r*dec_rise + in;  I += s - r
 *   AMPA: the same s, r; g = s - r;           I += g*(e_rev - v)
 * (dec = (float)exp(-dt/tau)); AMPA's inward current g*(e_rev - v) is the
 * declared I_syn = g*(V - E_rev) with the sign of current into the cell. */
enum { ORC_SYN_EXP = 1, ORC_SYN_DEXP = 2, ORC_SYN_AMPA = 3 };
#define ORC_MAX_CHAN 4

/* Number of model parameters, in this order:
 *  LIF : v_rest v_thresh v_reset tau_m tau_ref c_m i_bg                    (7)
 *  AdEx: v_rest v_thresh v_reset v_peak tau_m tau_w tau_ref c_m g_l a b
 *        delta_t i_bg                                                      (13)
 *  Izh : a b c d v_peak                                                    (5)
 * AdEx populations that receive conductance input additionally use
 *  cond[0..3] = tau_syn_exc, tau_syn_inh, e_exc, e_inh.                     */
#define ORC_NP_LIF 7
#define ORC_NP_ADEX 13
#define ORC_NP_IZH 5

typedef struct {
    int32_t model;
    int32_t n;
    int32_t offset;            /* global id of neuron 0 (drive counter key)  */
    int32_t drive_kind;
    double p[16];              /* uniform model parameters (SI / Izh units)  */
    double cond[4];            /* conductance synapse parameters (AdEx)      */
    double drive[4];           /* POISSON_*: lambda, amp; GAUSS: mean, std   */
    const float* init_v;       /* [n] or NULL (model default)                */
    const float* init_aux;     /* [n] w (AdEx) / u (Izh) or NULL             */
    const float* hp;           /* [np][n] per-neuron parameters or NULL      */
    int32_t n_chan;            /* synapse channels (0..ORC_MAX_CHAN)         */
    int32_t chan_kind[ORC_MAX_CHAN];
    double chan_tau[ORC_MAX_CHAN][2];   /* tau_rise, tau_decay (s)           */
    double chan_e[ORC_MAX_CHAN];        /* AMPA reversal potential            */
} orc_pop;

typedef struct {
    int32_t src_pop;
    int32_t tgt_pop;
    int32_t receptor;
    int32_t plastic;           /* 1: pair STDP attached                      */
    int64_t nnz;
    const int32_t* src;        /* [nnz] local source index (CSR order)       */
    const int32_t* tgt;        /* [nnz] local target index                   */
    const float* w;            /* [nnz] weight                               */
    const uint8_t* delay;      /* [nnz] delay in steps (>= 1)                */
    double stdp[7];            /* tau_plus tau_minus a_plus a_minus w_min w_max lr */
    float* w_out;              /* [nnz] final weights or NULL                */
} orc_proj;

typedef struct {
    int32_t npop;
    int32_t nproj;
    const orc_pop* pops;
    const orc_proj* projs;
    int32_t steps;
    int32_t slow_ratio;        /* plasticity runs when step % slow_ratio == 0 */
    double dt;
    uint64_t seed;
    /* outputs */
    int64_t spike_cap;
    int64_t* n_spikes;         /* [1] total spikes recorded                  */
    int32_t* spike_step;       /* [spike_cap]                                */
    int32_t* spike_id;         /* [spike_cap] global id, ascending per step  */
    float* final_v;            /* [N_total] or NULL                          */
    float* final_aux;          /* [N_total] or NULL                          */
    float* final_ref;          /* [N_total] or NULL                          */
    int32_t trace_n;           /* number of traced neurons                   */
    const int32_t* trace_ids;  /* [trace_n] global ids                       */
    float* trace_v;            /* [steps][trace_n] v after each step         */
    int32_t threads;           /* worker threads (harness: torch threads)    */
} orc_net;

/* ------------------------------------------------------------------------ */
/* 2. Philox4x32-10 and samplers                                            */
/* ------------------------------------------------------------------------ */

/* Stream identifiers (counter word 3) so that independent uses never share
 * a counter. */
enum {
    ORC_STREAM_DRIVE = 0x44524956u,   /* external drive, per (neuron, step) */
    ORC_STREAM_CONN = 0x434f4e4eu,    /* connectivity generation            */
    ORC_STREAM_INIT = 0x494e4954u     /* initial conditions / heterogeneity */
};

static inline void orc_philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
    const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
    const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
    for (int r = 0; r < 10; ++r) {
        uint64_t p0 = (uint64_t)M0 * c[0];
        uint64_t p1 = (uint64_t)M1 * c[2];
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        uint32_t n0 = hi1 ^ c[1] ^ k0;
        uint32_t n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
        k0 += W0; k1 += W1;
    }
}

/* Four 32-bit words for (seed, a, b, stream). */
static inline void orc_philox_words(uint64_t seed, uint32_t a, uint32_t b,
                                    uint32_t stream, uint32_t out[4]) {
    out[0] = a; out[1] = b; out[2] = 0u; out[3] = stream;
    orc_philox4x32_10(out, (uint32_t)seed, (uint32_t)(seed >> 32));
}

/* Uniform in (0,1): odd multiples of 2^-24, exact in binary32. */
static inline float orc_u01(uint32_t x) {
    return (float)(((x >> 9) << 1) | 1u) * 5.9604644775390625e-8f;
}

/* Poisson(lambda) by sequential inversion (Devroye 1986, X.3).  exp_neg_lam
 * is expf(-lambda) computed once on the host and passed in, so the device
 * and the oracle share it exactly.  Bounded at 255 events. */
static inline int orc_poisson(float u, float lam, float exp_neg_lam) {
    int k = 0;
    float p = exp_neg_lam;
    float F = p;
    while (u > F && k < 255) {
        k += 1;
        p = (p * lam) / (float)k;
        F = F + p;
    }
    return k;
}

/* ln(x) for normal x > 0: x = m * 2^e, m in [sqrt(1/2), sqrt(2)),
 * ln m = 2 atanh(s), s = (m-1)/(m+1), atanh series to s^11. */
static inline float orc_logf(float x) {
    union { float f; uint32_t u; } b;
    b.f = x;
    int e = (int)((b.u >> 23) & 0xffu) - 127;
    b.u = (b.u & 0x007fffffu) | 0x3f800000u;     /* m in [1,2) */
    float m = b.f;
    if (m > 1.41421353816986083984375f) { m = m * 0.5f; e += 1; }
    float s = (m - 1.0f) / (m + 1.0f);
    float s2 = s * s;
    float poly = 1.0f / 11.0f;
    poly = poly * s2 + 1.0f / 9.0f;
    poly = poly * s2 + 1.0f / 7.0f;
    poly = poly * s2 + 1.0f / 5.0f;
    poly = poly * s2 + 1.0f / 3.0f;
    poly = poly * s2 + 1.0f;
    float lnm = (2.0f * s) * poly;
    float fe = (float)e;
    /* ln 2 = LN2_HI + LN2_LO with LN2_HI exact in 16 bits. */
    return fe * 0.693145751953125f + (fe * 1.428606765330187045e-06f + lnm);
}

/* cos(2*pi*u) for u in [0,1): quadrant k = round(4u), r = u - k/4 in
 * [-1/8,1/8] (exact), x = 2*pi*r, Taylor series of sin/cos on [-pi/4,pi/4]. */
static inline float orc_cos2pi(float u) {
    float q = u * 4.0f;
    int k = (int)(q + 0.5f);
    float r = u - (float)k * 0.25f;
    float x = r * 6.28318548202514648438f;
    float x2 = x * x;
    float c = 1.0f / 40320.0f;
    c = c * x2 - 1.0f / 720.0f;
    c = c * x2 + 1.0f / 24.0f;
    c = c * x2 - 0.5f;
    c = c * x2 + 1.0f;
    float s = 1.0f / 362880.0f;
    s = s * x2 - 1.0f / 5040.0f;
    s = s * x2 + 1.0f / 120.0f;
    s = s * x2 - 1.0f / 6.0f;
    s = (s * x2) * x + x;
    switch (k & 3) {
        case 0: return c;
        case 1: return -s;
        case 2: return -c;
        default: return s;
    }
}

/* Standard normal from two uniforms (Box & Muller 1958). */
static inline float orc_normal(float u1, float u2) {
    float l = orc_logf(u1);
    float rad = sqrtf(-2.0f * l);
    return rad * orc_cos2pi(u2);
}

/* External drive of neuron gid at step: returns the amount added to the
 * current (kinds 1,2) or to the excitatory conductance input (kind 3).
 * Poisson kinds draw one uniform per neuron: word gid % 4 of the Philox
 * block (gid / 4, step), so four consecutive neurons share one block.  The
 * Gaussian kind uses words 0 and 1 of the block (gid, step). */
static inline float orc_drive_value(int kind, float d0, float d1, float exp_neg,
                                    uint64_t seed, uint32_t gid, uint32_t step) {
    uint32_t w[4];
    if (kind == ORC_DRIVE_POISSON_CURRENT || kind == ORC_DRIVE_POISSON_GEXC) {
        orc_philox_words(seed, gid >> 2, step, ORC_STREAM_DRIVE, w);
        int k = orc_poisson(orc_u01(w[gid & 3u]), d0, exp_neg);
        return d1 * (float)k;
    }
    orc_philox_words(seed, gid, step, ORC_STREAM_DRIVE, w);
    if (kind == ORC_DRIVE_GAUSS_CURRENT) {
        float z = orc_normal(orc_u01(w[0]), orc_u01(w[1]));
        return d0 + d1 * z;
    }
    return 0.0f;
}

/* ------------------------------------------------------------------------ */
/* 3. Neuron steps (fp32, reference operation order)                        */
/* ------------------------------------------------------------------------ */

/* LIF, src/neuron/lif.cpp:80-97.  Returns 1 on spike. */
static inline int orc_lif_step(float* v, float* ref, float I, float dt,
                               float v_rest, float v_thresh, float v_reset,
                               float tau_m, float tau_ref, float c_m, float i_bg) {
    int active = (*ref <= 0.0f);
    float r = (*ref > 0.0f) ? (*ref - dt) : *ref;
    float a = *v - v_rest;
    float lk = (-a) / tau_m;
    float in = (I + i_bg) / c_m;
    float dv = dt * (lk + in);
    float vn = active ? (*v + dv) : *v;
    int spiked = (vn >= v_thresh) && active;
    if (spiked) { vn = v_reset; r = tau_ref; }
    *v = vn;
    *ref = r;
    return spiked;
}

/* AdEx, src/neuron/adex.cpp:97-124.  expf stands in for torch::exp (the
 * reference's vectorised float exp; both are within ~1 ulp). */
static inline int orc_adex_step(float* v, float* w, float* ref, float I, float dt,
                                float v_rest, float v_thresh, float v_reset,
                                float v_peak, float tau_w, float tau_ref,
                                float c_m, float g_l, float a, float b,
                                float delta_t, float i_bg) {
    int active = (*ref <= 0.0f);
    float r = (*ref > 0.0f) ? (*ref - dt) : *ref;
    float vv = *v, ww = *w;
    float I_exp = (g_l * delta_t) * expf((vv - v_thresh) / delta_t);
    float acc = (-g_l) * (vv - v_rest);
    acc = acc + I_exp;
    acc = acc - ww;
    acc = acc + I;
    acc = acc + i_bg;
    float dv = (dt * acc) / c_m;
    float vn = active ? (vv + dv) : vv;
    float dw = (dt * ((a * (vn - v_rest)) - ww)) / tau_w;
    float wn = ww + dw;
    int spiked = (vn >= v_peak) && active;
    if (spiked) { vn = v_reset; wn = wn + b; r = tau_ref; }
    *v = vn; *w = wn; *ref = r;
    return spiked;
}

/* Izhikevich, src/neuron/izhikevich.cpp:76-98.  half = (float)(0.5*dt_ms),
 * dtm = (float)dt_ms with dt_ms = dt*1000 in double. */
static inline int orc_izh_step(float* v, float* u, float I, float half, float dtm,
                               float a, float b, float c, float d, float v_peak) {
    float vv = *v, uu = *u;
    float dv1 = (((0.04f * vv) * vv + 5.0f * vv) + 140.0f - uu) + I;
    vv = vv + half * dv1;
    float dv2 = (((0.04f * vv) * vv + 5.0f * vv) + 140.0f - uu) + I;
    vv = vv + half * dv2;
    float du = (dtm * a) * ((b * vv) - uu);
    uu = uu + du;
    int spiked = (vv >= v_peak);
    if (spiked) { vv = c; uu = uu + d; }
    *v = vv; *u = uu;
    return spiked;
}

/* Conductance synapse (AdEx population with g_exc/g_inh receptors):
 *   g <- g * exp(-dt/tau_syn) + input  (input delivered this step)
 *   I <- ((I + g_e*(E_e - v)) + g_i*(E_i - v))
 * The reference declares conductance synapses but never implements them
 * (src/synapse/exponential.cpp:37-42 throws), so this step is defined here. */
static inline float orc_cond_current(float I, float* ge, float* gi, float in_e,
                                     float in_i, float dec_e, float dec_i,
                                     float e_exc, float e_inh, float v) {
    float g_e = (*ge * dec_e) + in_e;
    float g_i = (*gi * dec_i) + in_i;
    *ge = g_e; *gi = g_i;
    float r = I + g_e * (e_exc - v);
    r = r + g_i * (e_inh - v);
    return r;
}

/* exp(-x) and log(u) that give the same bits on every platform (the
 * device generators use the same method): only IEEE double +, -, *, / and
 * exact scaling by powers of two.  exp(-x): Cody and Waite's reduction
 * x = k ln2 + r (ln2 split into an exact high part and a low part), then
 * 22 Taylor terms of exp(-r); log(u): u = m 2^e, ln m = 2 atanh((m-1)/(m+1))
 * by its series to the 45th power, plus e ln2. */
static inline double orc_exp_neg(double x) {
    if (!(x > 0.0)) return 1.0;
    if (x > 745.0) return 0.0;
    const double lh = 6.93147180369123816490e-01, ll = 1.90821492927058770002e-10;
    const double k = floor(x / 6.93147180559945309417e-01);
    const double r = (x - k * lh) - k * ll;
    double s = 1.0;
    for (int i = 22; i >= 1; --i) s = 1.0 - (r / (double)i) * s;
    return ldexp(s, -(int)k);
}

static inline double orc_log(double u) {
    int e = 0;
    const double m = frexp(u, &e);
    const double z = (m - 1.0) / (m + 1.0);
    const double z2 = z * z;
    double s = 0.0;
    for (int i = 45; i >= 3; i -= 2) s = (s + 1.0 / (double)i) * z2;
    return 2.0 * z * (1.0 + s) + (double)e * 6.93147180559945309417e-01;
}

/* One synapse channel of one neuron (see ORC_SYN_*): returns I plus the
 * channel's current; s (decay state) and r (rise state) updated. */
static inline float orc_chan_current(int kind, float I, float* s, float* r, float in, float dec_rise,
                                     float dec_decay, float e_rev, float v) {
    float sd = (*s * dec_decay) + in;
    *s = sd;
    if (kind == ORC_SYN_EXP) return I + sd;
    float sr = (*r * dec_rise) + in;
    *r = sr;
    float g = sd - sr;
    if (kind == ORC_SYN_DEXP) return I + g;
    return I + g * (e_rev - v);
}

#ifdef __cplusplus
}
#endif
#endif /* NRN_ORACLE_COMMON_H */
