/*
 * nrn_oracle.c -- CPU restatement of libnrn's per-timestep hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker).  The product never links or calls
 * this file.  It is pinned against outputs of the reference itself, compiled
 * from its own sources (oracle/Makefile, ref_harness.cpp), through the golden
 * fixtures under tests/golden/.
 *
 * One step follows the phase order of the reference's sim_step
 * (src/simulation/runner.cpp:95-173):
 *   P1 zero the synaptic input of every population           (:99-104)
 *   P2 deliver, for every projection, the spikes emitted d steps ago through
 *      each synapse of delay d (the reference reads SpikeBuffer::read(1),
 *      src/simulation/spike_buffer.cpp:32-49; per-synapse delays are the
 *      extension the reference's ConnectivityTensor::delays declares but
 *      sim_step never reads, runner.cpp:113)                 (:106-124)
 *      + external drive (Philox; the reference has none)
 *   P3 neuron update (oracle_common.h, one function per model)(:127-129)
 *   P4 push spikes into the history                          (:131-139)
 *   P5 pair STDP at slow-clock boundaries, src/plasticity/stdp.cpp:43-141,
 *      restated per neuron trace (the reference's per-synapse traces are
 *      identical along each row/column, stdp.cpp:118-128)    (:142-150)
 *   P6 spike recording, ascending ids, src/monitor/spike_recorder.cpp:33-58
 * Before the first step every population runs one update with dt = 0, as
 * sim_create does (runner.cpp:36-38).
 *
 * Delivery sums each target's input in CSR order (projection, then source,
 * then synapse); the reference sums per 64..256-wide block with BLAS sgemv.
 * Both are fp32; they agree exactly when the weights are dyadic rationals
 * whose partial sums are exact, and to rounding otherwise.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>

#include "oracle_common.h"

#define ORC_EXPORT __attribute__((visibility("default")))

static int model_np(int model) {
    return model == ORC_LIF ? ORC_NP_LIF : model == ORC_ADEX ? ORC_NP_ADEX : ORC_NP_IZH;
}

/* Parameter k of neuron i: per-neuron array when given, else uniform. */
static inline float par(const orc_pop* P, int k, int i) {
    return P->hp ? P->hp[(size_t)k * P->n + i] : (float)P->p[k];
}

typedef struct {
    float* v;
    float* aux;     /* w (AdEx) or u (Izh) */
    float* ref;
    float* ge;      /* conductances (AdEx with conductance input) */
    float* gi;
    int cond;       /* population receives conductance input */
    float* cs[ORC_MAX_CHAN];   /* synapse channel decay state */
    float* cr[ORC_MAX_CHAN];   /* synapse channel rise state  */
} pop_state;

static void init_pop(const orc_pop* P, pop_state* S) {
    int n = P->n;
    S->v = (float*)calloc((size_t)n, sizeof(float));
    S->aux = (float*)calloc((size_t)n, sizeof(float));
    S->ref = (float*)calloc((size_t)n, sizeof(float));
    S->ge = (float*)calloc((size_t)n, sizeof(float));
    S->gi = (float*)calloc((size_t)n, sizeof(float));
    for (int c = 0; c < ORC_MAX_CHAN; ++c) {
        S->cs[c] = (float*)calloc((size_t)n, sizeof(float));
        S->cr[c] = (float*)calloc((size_t)n, sizeof(float));
    }
    for (int i = 0; i < n; ++i) {
        float v0, a0 = 0.0f;
        if (P->model == ORC_IZH) {
            /* izh_create: v = v_init, u = b*v_init (double product, then
             * float), src/neuron/izhikevich.cpp:45-46; v_init = -65. */
            v0 = -65.0f;
            a0 = (float)(P->p[1] * -65.0);
        } else {
            v0 = (float)P->p[0];   /* v_rest */
        }
        S->v[i] = P->init_v ? P->init_v[i] : v0;
        S->aux[i] = P->init_aux ? P->init_aux[i] : a0;
    }
}

static void free_pop(pop_state* S) {
    free(S->v); free(S->aux); free(S->ref); free(S->ge); free(S->gi);
    for (int c = 0; c < ORC_MAX_CHAN; ++c) { free(S->cs[c]); free(S->cr[c]); }
}

/* This step's synapse channel currents added to the input of every neuron
 * (before the model update); cin[c] is channel c's input, or NULL. */
static void apply_channels(const orc_pop* P, pop_state* S, float* I, float* const* cin, double dt) {
    for (int c = 0; c < P->n_chan && c < ORC_MAX_CHAN; ++c) {
        float dr = (float)exp(-dt / P->chan_tau[c][0]);
        float dd = (float)exp(-dt / P->chan_tau[c][1]);
        float e = (float)P->chan_e[c];
        for (int i = 0; i < P->n; ++i)
            I[i] = orc_chan_current(P->chan_kind[c], I[i], &S->cs[c][i], &S->cr[c][i],
                                    cin && cin[c] ? cin[c][i] : 0.0f, dr, dd, e, S->v[i]);
    }
}

/* One update of population P with per-neuron inputs I[], conductance
 * inputs ie[]/ii[] (may be NULL), step length dt; spk[] receives 0/1. */
static void update_pop(const orc_pop* P, pop_state* S, const float* I,
                       const float* ie, const float* ii, double dt, uint8_t* spk) {
    int n = P->n;
    float dtf = (float)dt;
    if (P->model == ORC_LIF) {
        for (int i = 0; i < n; ++i) {
            spk[i] = (uint8_t)orc_lif_step(&S->v[i], &S->ref[i], I[i], dtf,
                par(P, 0, i), par(P, 1, i), par(P, 2, i), par(P, 3, i),
                par(P, 4, i), par(P, 5, i), par(P, 6, i));
        }
    } else if (P->model == ORC_ADEX) {
        float dec_e = 1.0f, dec_i = 1.0f;
        if (S->cond) {
            dec_e = (float)exp(-dt / P->cond[0]);
            dec_i = (float)exp(-dt / P->cond[1]);
        }
        for (int i = 0; i < n; ++i) {
            float Ii = I[i];
            if (S->cond) {
                Ii = orc_cond_current(Ii, &S->ge[i], &S->gi[i], ie ? ie[i] : 0.0f,
                                      ii ? ii[i] : 0.0f, dec_e, dec_i,
                                      (float)P->cond[2], (float)P->cond[3], S->v[i]);
            }
            spk[i] = (uint8_t)orc_adex_step(&S->v[i], &S->aux[i], &S->ref[i], Ii, dtf,
                par(P, 0, i), par(P, 1, i), par(P, 2, i), par(P, 3, i),
                par(P, 5, i), par(P, 6, i), par(P, 7, i), par(P, 8, i),
                par(P, 9, i), par(P, 10, i), par(P, 11, i), par(P, 12, i));
        }
    } else {
        double dt_ms = dt * 1000.0;
        float half = (float)(0.5 * dt_ms);
        float dtm = (float)dt_ms;
        for (int i = 0; i < n; ++i) {
            spk[i] = (uint8_t)orc_izh_step(&S->v[i], &S->aux[i], I[i], half, dtm,
                par(P, 0, i), par(P, 1, i), par(P, 2, i), par(P, 3, i), par(P, 4, i));
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Neuron-only run: per-step input currents, as the reference's neuron tests */
/* call *_forward directly (tests/neuron/test_neuron_dynamics.cpp:24-232).   */
/* ------------------------------------------------------------------------ */
ORC_EXPORT int orc_neuron_run(const orc_pop* P, int steps, double dt,
                              const float* I /* [steps][n] or NULL */,
                              float* out_v, float* out_aux, float* out_ref,
                              uint8_t* out_spike /* each [steps][n] or NULL */) {
    pop_state S;
    memset(&S, 0, sizeof(S));
    init_pop(P, &S);
    int n = P->n;
    float* zero = (float*)calloc((size_t)n, sizeof(float));
    uint8_t* spk = (uint8_t*)calloc((size_t)n, 1);
    for (int t = 0; t < steps; ++t) {
        const float* It = I ? I + (size_t)t * n : zero;
        update_pop(P, &S, It, NULL, NULL, dt, spk);
        size_t o = (size_t)t * n;
        if (out_v) memcpy(out_v + o, S.v, (size_t)n * sizeof(float));
        if (out_aux) memcpy(out_aux + o, S.aux, (size_t)n * sizeof(float));
        if (out_ref) memcpy(out_ref + o, S.ref, (size_t)n * sizeof(float));
        if (out_spike) memcpy(out_spike + o, spk, (size_t)n);
    }
    free(zero); free(spk); free_pop(&S);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Network run                                                              */
/* ------------------------------------------------------------------------ */
ORC_EXPORT int orc_net_run(const orc_net* net) {
    int np = net->npop, nq = net->nproj;
    int64_t N = 0;
    for (int p = 0; p < np; ++p) {
        if (net->pops[p].offset != N) return -1;   /* offsets must be dense */
        N += net->pops[p].n;
    }
    int maxd = 1;
    for (int q = 0; q < nq; ++q) {
        const orc_proj* Q = &net->projs[q];
        for (int64_t k = 0; k < Q->nnz; ++k) {
            if (Q->delay[k] < 1) return -2;
            if (Q->delay[k] > maxd) maxd = Q->delay[k];
        }
    }
    int H = maxd + 1;

    pop_state* S = (pop_state*)calloc((size_t)np, sizeof(pop_state));
    for (int p = 0; p < np; ++p) init_pop(&net->pops[p], &S[p]);
    for (int q = 0; q < nq; ++q) {
        if (net->projs[q].receptor == ORC_RECV_GEXC || net->projs[q].receptor == ORC_RECV_GINH)
            S[net->projs[q].tgt_pop].cond = 1;
    }
    for (int p = 0; p < np; ++p)
        if (net->pops[p].drive_kind == ORC_DRIVE_POISSON_GEXC) S[p].cond = 1;

    float* I = (float*)calloc((size_t)N, sizeof(float));
    float* ie = (float*)calloc((size_t)N, sizeof(float));
    float* ii = (float*)calloc((size_t)N, sizeof(float));
    /* synapse channel inputs, global-id indexed per channel slot */
    float* cin_all[ORC_MAX_CHAN];
    for (int c = 0; c < ORC_MAX_CHAN; ++c) cin_all[c] = (float*)calloc((size_t)N, sizeof(float));
    uint8_t* hist = (uint8_t*)calloc((size_t)H * N, 1);

    /* Event-driven indices: per projection, synapse positions ordered by
     * (source, delay, list position) with row offsets per source, and for
     * plastic projections the synapses of every target. */
    int64_t** row = (int64_t**)calloc((size_t)(nq > 0 ? nq : 1), sizeof(int64_t*));
    int64_t** perm = (int64_t**)calloc((size_t)(nq > 0 ? nq : 1), sizeof(int64_t*));
    int64_t** inrow = (int64_t**)calloc((size_t)(nq > 0 ? nq : 1), sizeof(int64_t*));
    int64_t** inlist = (int64_t**)calloc((size_t)(nq > 0 ? nq : 1), sizeof(int64_t*));
    int* first_stdp = (int*)calloc((size_t)(nq > 0 ? nq : 1), sizeof(int));
    for (int q = 0; q < nq; ++q) {
        const orc_proj* Q = &net->projs[q];
        int ns = net->pops[Q->src_pop].n, nt = net->pops[Q->tgt_pop].n;
        int64_t* cnt = (int64_t*)calloc((size_t)ns * 256 + 1, sizeof(int64_t));
        for (int64_t k = 0; k < Q->nnz; ++k) cnt[(size_t)Q->src[k] * 256 + Q->delay[k] + 1]++;
        for (size_t b = 0; b < (size_t)ns * 256; ++b) cnt[b + 1] += cnt[b];
        perm[q] = (int64_t*)malloc((size_t)(Q->nnz > 0 ? Q->nnz : 1) * sizeof(int64_t));
        row[q] = (int64_t*)malloc(((size_t)ns + 1) * sizeof(int64_t));
        for (int j = 0; j <= ns; ++j) row[q][j] = cnt[(size_t)j * 256];
        for (int64_t k = 0; k < Q->nnz; ++k) perm[q][cnt[(size_t)Q->src[k] * 256 + Q->delay[k]]++] = k;
        free(cnt);
        first_stdp[q] = 1;
        if (Q->plastic) {
            int64_t* c2 = (int64_t*)calloc((size_t)nt + 1, sizeof(int64_t));
            for (int64_t k = 0; k < Q->nnz; ++k) c2[Q->tgt[k] + 1]++;
            for (int i = 0; i < nt; ++i) c2[i + 1] += c2[i];
            inrow[q] = (int64_t*)malloc(((size_t)nt + 1) * sizeof(int64_t));
            memcpy(inrow[q], c2, ((size_t)nt + 1) * sizeof(int64_t));
            inlist[q] = (int64_t*)malloc((size_t)(Q->nnz > 0 ? Q->nnz : 1) * sizeof(int64_t));
            for (int64_t k = 0; k < Q->nnz; ++k) inlist[q][c2[Q->tgt[k]]++] = k;
            free(c2);
        }
    }
    /* newest spike step of every neuron (delivery skips silent sources) */
    int32_t* last = (int32_t*)malloc((size_t)N * sizeof(int32_t));
    for (int64_t g = 0; g < N; ++g) last[g] = -1000000;

    /* Working copies of the weights and STDP traces. */
    float** W = (float**)calloc((size_t)(nq > 0 ? nq : 1), sizeof(float*));
    float** xpre = (float**)calloc((size_t)(nq > 0 ? nq : 1), sizeof(float*));
    float** xpost = (float**)calloc((size_t)(nq > 0 ? nq : 1), sizeof(float*));
    for (int q = 0; q < nq; ++q) {
        const orc_proj* Q = &net->projs[q];
        W[q] = (float*)malloc((size_t)(Q->nnz > 0 ? Q->nnz : 1) * sizeof(float));
        memcpy(W[q], Q->w, (size_t)Q->nnz * sizeof(float));
        if (Q->plastic) {
            xpre[q] = (float*)calloc((size_t)net->pops[Q->src_pop].n, sizeof(float));
            xpost[q] = (float*)calloc((size_t)net->pops[Q->tgt_pop].n, sizeof(float));
        }
    }

    /* sim_create: one update with dt = 0 and zero input; not recorded. */
    for (int p = 0; p < np; ++p) {
        const orc_pop* P = &net->pops[p];
        update_pop(P, &S[p], I + P->offset, ie + P->offset, ii + P->offset, 0.0,
                   hist + P->offset /* scratch, cleared below */);
    }
    memset(hist, 0, (size_t)H * N);

    int64_t nspk = 0;
    int slow = net->slow_ratio > 0 ? net->slow_ratio : 1;
    for (int t = 0; t < net->steps; ++t) {
        /* P1 */
        memset(I, 0, (size_t)N * sizeof(float));
        memset(ie, 0, (size_t)N * sizeof(float));
        memset(ii, 0, (size_t)N * sizeof(float));
        for (int c = 0; c < ORC_MAX_CHAN; ++c) memset(cin_all[c], 0, (size_t)N * sizeof(float));
        /* P2: arrival-time delivery with the weights as they are now. */
        for (int q = 0; q < nq; ++q) {
            const orc_proj* Q = &net->projs[q];
            int so = net->pops[Q->src_pop].offset, to = net->pops[Q->tgt_pop].offset;
            float* acc = Q->receptor >= ORC_RECV_CHANNEL ? cin_all[(Q->receptor - ORC_RECV_CHANNEL) % ORC_MAX_CHAN]
                       : Q->receptor == ORC_RECV_CURRENT ? I
                       : Q->receptor == ORC_RECV_GEXC ? ie : ii;
            /* per target: sources ascending, then delay, then list position */
            int ns = net->pops[Q->src_pop].n;
            for (int j = 0; j < ns; ++j) {
                if (last[so + j] < t - maxd) continue;
                for (int64_t r = row[q][j]; r < row[q][j + 1]; ++r) {
                    int64_t k = perm[q][r];
                    int d = Q->delay[k];
                    if (t - d < 0) continue;
                    if (hist[(size_t)((t - d) % H) * N + so + j])
                        acc[to + Q->tgt[k]] += W[q][k];
                }
            }
        }
        /* external drive */
        for (int p = 0; p < np; ++p) {
            const orc_pop* P = &net->pops[p];
            if (P->drive_kind == ORC_DRIVE_NONE) continue;
            float d0 = (float)P->drive[0], d1 = (float)P->drive[1];
            float en = (float)exp(-P->drive[0]);
            float* dst = P->drive_kind == ORC_DRIVE_POISSON_GEXC ? ie : I;
            for (int i = 0; i < P->n; ++i) {
                uint32_t gid = (uint32_t)(P->offset + i);
                dst[gid] += orc_drive_value(P->drive_kind, d0, d1, en, net->seed, gid,
                                            (uint32_t)t);
            }
        }
        /* P3 + P4 */
        uint8_t* h = hist + (size_t)(t % H) * N;
        for (int p = 0; p < np; ++p) {
            const orc_pop* P = &net->pops[p];
            float* cin[ORC_MAX_CHAN];
            for (int c = 0; c < ORC_MAX_CHAN; ++c) cin[c] = cin_all[c] + P->offset;
            apply_channels(P, &S[p], I + P->offset, cin, net->dt);
            update_pop(P, &S[p], I + P->offset, ie + P->offset, ii + P->offset,
                       net->dt, h + P->offset);
        }
        /* P5: STDP (stdp.cpp:43-141), every synapse, every slow boundary. */
        if (t % slow == 0) {
            for (int q = 0; q < nq; ++q) {
                const orc_proj* Q = &net->projs[q];
                if (!Q->plastic) continue;
                const orc_pop* Ps = &net->pops[Q->src_pop];
                const orc_pop* Pt = &net->pops[Q->tgt_pop];
                const uint8_t* pre = h + Ps->offset;
                const uint8_t* post = h + Pt->offset;
                float dpre = (float)exp(-net->dt / Q->stdp[0]);
                float dpost = (float)exp(-net->dt / Q->stdp[1]);
                float ap = (float)Q->stdp[2];
                float am = (float)fabs(Q->stdp[3]);
                float wmin = (float)Q->stdp[4], wmax = (float)Q->stdp[5];
                float lr = (float)Q->stdp[6];
                for (int j = 0; j < Ps->n; ++j)
                    xpre[q][j] = xpre[q][j] * dpre + (float)pre[j];
                for (int i = 0; i < Pt->n; ++i)
                    xpost[q][i] = xpost[q][i] * dpost + (float)post[i];
                /* Every synapse is updated (and clamped) at the first update;
                 * afterwards only synapses whose source or target spiked can
                 * change (dw = 0 otherwise, the weight already in range), so
                 * only those are visited: the out-rows of spiking sources,
                 * then the in-lists of spiking targets whose source did not. */
#define ORC_STDP_SYN(k)                                                          \
    do {                                                                         \
        int j_ = Q->src[k], i_ = Q->tgt[k];                                      \
        float dw = (ap * xpre[q][j_]) * (float)post[i_]                          \
                 - (am * xpost[q][i_]) * (float)pre[j_];                         \
        float wn = W[q][k] + ((dw * lr) * 1.0f) * 1.0f;                          \
        if (wn < wmin) wn = wmin;                                                \
        if (wn > wmax) wn = wmax;                                                \
        W[q][k] = wn;                                                            \
    } while (0)
                if (first_stdp[q]) {
                    for (int64_t k = 0; k < Q->nnz; ++k) ORC_STDP_SYN(k);
                    first_stdp[q] = 0;
                } else {
                    for (int j = 0; j < Ps->n; ++j) {
                        if (!pre[j]) continue;
                        for (int64_t r = row[q][j]; r < row[q][j + 1]; ++r) ORC_STDP_SYN(perm[q][r]);
                    }
                    for (int i = 0; i < Pt->n; ++i) {
                        if (!post[i]) continue;
                        for (int64_t r = inrow[q][i]; r < inrow[q][i + 1]; ++r) {
                            int64_t k = inlist[q][r];
                            if (!pre[Q->src[k]]) ORC_STDP_SYN(k);
                        }
                    }
                }
#undef ORC_STDP_SYN
            }
        }
        /* P6 */
        for (int64_t g = 0; g < N; ++g) {
            if (!h[g]) continue;
            last[g] = t;
            if (nspk < net->spike_cap) {
                net->spike_step[nspk] = t;
                net->spike_id[nspk] = (int32_t)g;
            }
            ++nspk;
        }
        if (net->trace_n > 0 && net->trace_v) {
            for (int k = 0; k < net->trace_n; ++k) {
                int32_t g = net->trace_ids[k];
                int p = 0;
                while (p + 1 < np && net->pops[p + 1].offset <= g) ++p;
                net->trace_v[(size_t)t * net->trace_n + k] = S[p].v[g - net->pops[p].offset];
            }
        }
    }
    if (net->n_spikes) *net->n_spikes = nspk;

    for (int p = 0; p < np; ++p) {
        const orc_pop* P = &net->pops[p];
        if (net->final_v) memcpy(net->final_v + P->offset, S[p].v, (size_t)P->n * 4);
        if (net->final_aux) memcpy(net->final_aux + P->offset, S[p].aux, (size_t)P->n * 4);
        if (net->final_ref) memcpy(net->final_ref + P->offset, S[p].ref, (size_t)P->n * 4);
    }
    for (int q = 0; q < nq; ++q) {
        const orc_proj* Q = &net->projs[q];
        if (Q->w_out) memcpy(Q->w_out, W[q], (size_t)Q->nnz * sizeof(float));
        free(W[q]); free(xpre[q]); free(xpost[q]);
    }
    free(W); free(xpre); free(xpost);
    for (int p = 0; p < np; ++p) free_pop(&S[p]);
    for (int q = 0; q < nq; ++q) { free(row[q]); free(perm[q]); free(inrow[q]); free(inlist[q]); }
    free(row); free(perm); free(inrow); free(inlist); free(first_stdp); free(last);
    free(S); free(I); free(ie); free(ii); free(hist);
    for (int c = 0; c < ORC_MAX_CHAN; ++c) free(cin_all[c]);
    return nspk > net->spike_cap ? 1 : 0;
}

/* ------------------------------------------------------------------------ */
/* Connectivity generators (the reference has Erdos-Renyi only,             */
/* src/connectivity/topology/random.cpp:25-95; fixed in/out-degree are      */
/* defined here and on the device with the same Philox stream).             */
/*                                                                          */
/* A draw belongs to (row r, slot k) of generator `gen`; rows are targets   */
/* (fixed in-degree) or sources (fixed out-degree), identified by global    */
/* id g_r = row_offset + r:                                                 */
/*   words  = Philox(seed; c0 = g_r, c1 = k, c2 = gen, c3 = ORC_STREAM_CONN) */
/*   column = (w0 * m) >> 32 over the m = n_col candidate columns, or over  */
/*            n_col - 1 when autapses are excluded and g_r lies inside the  */
/*            column range, the draw then skipping g_r's own column         */
/*   delay  = dmin + ((w1 * (dmax-dmin+1)) >> 32)                           */
/*   weight = w_lo + w_span * u01(w2)                                       */
/* Only synapses whose target global id lies in [keep_lo, keep_hi) are      */
/* kept (one draw stream can feed several target populations).  Synapses   */
/* are emitted source-major, ties in (row, slot) order (a stable sort).     */
/* ------------------------------------------------------------------------ */
static inline void conn_words(uint64_t seed, uint32_t c0, uint32_t c1, uint32_t c2,
                              uint32_t w[4]) {
    w[0] = c0; w[1] = c1; w[2] = c2; w[3] = ORC_STREAM_CONN;
    orc_philox4x32_10(w, (uint32_t)seed, (uint32_t)(seed >> 32));
}

/* Returns the number of synapses written (source/target as local indices of
 * the source range and of the kept target range), or the count alone when
 * the output pointers are NULL. */
ORC_EXPORT int64_t orc_gen_fixed_degree(
    int out_degree_mode, uint64_t seed, uint32_t gen,
    int32_t n_src, int32_t src_offset, int32_t n_tgt, int32_t tgt_offset,
    int32_t degree, int autapses_excluded, int32_t dmin, int32_t dmax,
    float w_lo, float w_span, int32_t keep_lo, int32_t keep_hi,
    int32_t* out_src, int32_t* out_tgt, float* out_w, uint8_t* out_delay) {
    int32_t nrow = out_degree_mode ? n_src : n_tgt;
    int32_t ncol = out_degree_mode ? n_tgt : n_src;
    int32_t roff = out_degree_mode ? src_offset : tgt_offset;
    int32_t coff = out_degree_mode ? tgt_offset : src_offset;
    int64_t total = (int64_t)nrow * degree;
    int32_t* s = (int32_t*)malloc((size_t)(total > 0 ? total : 1) * 4);
    int32_t* tg = (int32_t*)malloc((size_t)(total > 0 ? total : 1) * 4);
    float* ww = (float*)malloc((size_t)(total > 0 ? total : 1) * 4);
    uint8_t* dd = (uint8_t*)malloc((size_t)(total > 0 ? total : 1));
    uint32_t span = (uint32_t)(dmax - dmin + 1);
    int64_t e = 0;
    for (int32_t r = 0; r < nrow; ++r) {
        int32_t g = roff + r;
        int self = autapses_excluded && g >= coff && g < coff + ncol;
        uint32_t m = (uint32_t)(self ? ncol - 1 : ncol);
        for (int32_t k = 0; k < degree; ++k) {
            uint32_t w[4];
            conn_words(seed, (uint32_t)g, (uint32_t)k, gen, w);
            uint32_t c = (uint32_t)(((uint64_t)w[0] * m) >> 32);
            if (self && c >= (uint32_t)(g - coff)) c += 1;
            uint32_t d = (uint32_t)dmin + (uint32_t)(((uint64_t)w[1] * span) >> 32);
            int32_t src_g = out_degree_mode ? g : coff + (int32_t)c;
            int32_t tgt_g = out_degree_mode ? coff + (int32_t)c : g;
            if (tgt_g < keep_lo || tgt_g >= keep_hi) continue;
            s[e] = src_g - src_offset;
            tg[e] = tgt_g - keep_lo;
            ww[e] = w_lo + w_span * orc_u01(w[2]);
            dd[e] = (uint8_t)d;
            ++e;
        }
    }
    if (out_src) {
        /* stable counting sort by source */
        int64_t* cnt = (int64_t*)calloc((size_t)n_src + 1, sizeof(int64_t));
        for (int64_t k = 0; k < e; ++k) cnt[s[k] + 1]++;
        for (int32_t j = 0; j < n_src; ++j) cnt[j + 1] += cnt[j];
        for (int64_t k = 0; k < e; ++k) {
            int64_t pos = cnt[s[k]]++;
            out_src[pos] = s[k]; out_tgt[pos] = tg[k]; out_w[pos] = ww[k]; out_delay[pos] = dd[k];
        }
        free(cnt);
    }
    free(s); free(tg); free(ww); free(dd);
    return e;
}

/* Per-neuron initial values: lo + span * u01(Philox(seed; gid, which, 0,
 * ORC_STREAM_INIT)[0]). */
ORC_EXPORT void orc_init_uniform(uint64_t seed, uint32_t which, int32_t offset, int32_t n,
                                 float lo, float span, float* out) {
    for (int32_t i = 0; i < n; ++i) {
        uint32_t w[4] = {(uint32_t)(offset + i), which, 0u, ORC_STREAM_INIT};
        orc_philox4x32_10(w, (uint32_t)seed, (uint32_t)(seed >> 32));
        out[i] = lo + span * orc_u01(w[0]);
    }
}

/* Drive samples, for checking the device RNG. */
ORC_EXPORT void orc_drive_values(int kind, double d0, double d1, uint64_t seed,
                                 int32_t offset, int32_t n, int32_t step, float* out) {
    float en = (float)exp(-d0);
    for (int i = 0; i < n; ++i)
        out[i] = orc_drive_value(kind, (float)d0, (float)d1, en, seed,
                                 (uint32_t)(offset + i), (uint32_t)step);
}

ORC_EXPORT void orc_philox(uint64_t seed, uint32_t c0, uint32_t c1, uint32_t c2,
                           uint32_t c3, uint32_t* out4) {
    out4[0] = c0; out4[1] = c1; out4[2] = c2; out4[3] = c3;
    orc_philox4x32_10(out4, (uint32_t)seed, (uint32_t)(seed >> 32));
}

ORC_EXPORT float orc_normal_from_words(uint32_t a, uint32_t b) {
    return orc_normal(orc_u01(a), orc_u01(b));
}

/* ------------------------------------------------------------------------ */
/* Random and distance-dependent connectivity, restating the rules of the   */
/* reference's random (src/connectivity/topology/random.cpp:25-95: each     */
/* pair with probability p, autapses removed) and distance-dependent        */
/* (src/connectivity/topology/distance_dependent.cpp:28-144: 1D positions   */
/* i * L / n, p = max(exp(-d^2 / 2 sigma^2), p_min)) topologies with the    */
/* Philox draws of the device generators: per target row g (global id),     */
/*   ER: geometric skips, gap = floor(ln u / ln(1 - p)),                    */
/*       u = (Philox(seed; g, draw, gen, ER)[0] + 0.5) / 2^32;              */
/*   distance: pair (t, s) iff Philox(seed; g, s/4, gen, DIST)[s%4]         */
/*       < floor(p 2^32);                                                    */
/*   delay and weight of the k-th synapse of the row from                   */
/*       Philox(seed; g, k, gen, SYN): dmin + (w0 * span >> 32),            */
/*       w_lo + w_span * u01(w1).                                            */
/* Rows are target population indices [tgt_lo, tgt_lo + n_rows); synapses   */
/* are emitted row by row, sources ascending.  Returns the count (outputs   */
/* may be NULL to count).                                                    */
/* ------------------------------------------------------------------------ */
#define ORC_STREAM_ER 0x45524E44u
#define ORC_STREAM_DIST 0x44495354u
#define ORC_STREAM_SYN 0x53594E31u

static inline uint32_t orc_prob_threshold(double p) {
    if (!(p > 0.0)) return 0u;
    double t = floor(p * 4294967296.0);
    return t >= 4294967295.0 ? 0xFFFFFFFFu : (uint32_t)t;
}

ORC_EXPORT int64_t orc_gen_random(int rule, uint64_t seed, uint32_t gen, int32_t n_src, int32_t n_tgt,
                                  int32_t tgt_lo, int32_t n_rows, int32_t tgt_gid_offset, int same_pop,
                                  double p, double sigma, double max_distance, double p_min,
                                  int32_t dmin, int32_t dmax, float w_lo, float w_span,
                                  int32_t* out_src, int32_t* out_tgt, float* out_w, uint8_t* out_delay) {
    int64_t e = 0;
    uint32_t span = (uint32_t)(dmax - dmin + 1);
    double log1mp = p < 1.0 ? orc_log(1.0 - p) : 0.0;
    double sp_s = n_src > 1 ? max_distance / n_src : 0.0, sp_t = n_tgt > 1 ? max_distance / n_tgt : 0.0;
    double inv2s2 = rule == 2 ? 1.0 / (2.0 * sigma * sigma) : 0.0;
    for (int32_t r = 0; r < n_rows; ++r) {
        int32_t t = tgt_lo + r;
        uint32_t g = (uint32_t)(tgt_gid_offset + t);
        int32_t self = same_pop ? t : -1;
        uint32_t k = 0;
        /* emits source s as the row's k-th synapse */
#define ORC_EMIT(s)                                                              \
    do {                                                                         \
        if (out_src) {                                                           \
            uint32_t y[4];                                                       \
            y[0] = g; y[1] = k; y[2] = gen; y[3] = ORC_STREAM_SYN;               \
            orc_philox4x32_10(y, (uint32_t)seed, (uint32_t)(seed >> 32));        \
            out_src[e] = (s);                                                    \
            out_tgt[e] = r;                                                      \
            out_delay[e] = (uint8_t)((uint32_t)dmin + (uint32_t)(((uint64_t)y[0] * span) >> 32)); \
            out_w[e] = w_lo + w_span * orc_u01(y[1]);                            \
        }                                                                        \
        ++e;                                                                     \
        ++k;                                                                     \
    } while (0)
        if (rule == 1) {
            if (!(p > 0.0)) continue;
            int64_t pos = -1;
            for (uint32_t draw = 0;; ++draw) {
                int64_t step = 1;
                if (p < 1.0) {
                    uint32_t x[4] = {g, draw, gen, ORC_STREAM_ER};
                    orc_philox4x32_10(x, (uint32_t)seed, (uint32_t)(seed >> 32));
                    double u = ((double)x[0] + 0.5) * (1.0 / 4294967296.0);
                    double l = orc_log(u);
                    if (l > 0.0) l = 0.0;
                    double gap = floor(l / log1mp);
                    if (gap >= (double)n_src) break;
                    step = 1 + (int64_t)gap;
                }
                pos += step;
                if (pos >= n_src) break;
                if (pos != self) ORC_EMIT((int32_t)pos);
            }
        } else {
            double xt = (double)t * sp_t;
            int64_t s0 = 0, s1 = n_src;
            if (!(p_min > 0.0) && sp_s > 0.0) {
                double hw = sigma * sqrt(2.0 * 40.0 * 6.93147180559945309417e-01);
                double lo = floor((xt - hw) / sp_s), hi = ceil((xt + hw) / sp_s) + 1.0;
                s0 = lo < 0.0 ? 0 : (int64_t)lo;
                s1 = hi > (double)n_src ? n_src : (int64_t)hi;
            }
            uint32_t x[4] = {0, 0, 0, 0};
            for (int64_t s = s0; s < s1; ++s) {
                if ((s & 3) == 0 || s == s0) {
                    x[0] = g; x[1] = (uint32_t)(s >> 2); x[2] = gen; x[3] = ORC_STREAM_DIST;
                    orc_philox4x32_10(x, (uint32_t)seed, (uint32_t)(seed >> 32));
                }
                if (s == self) continue;
                double d = xt - (double)s * sp_s;
                double pp = orc_exp_neg((d * d) * inv2s2);
                if (pp < p_min) pp = p_min;
                if (x[s & 3] < orc_prob_threshold(pp)) ORC_EMIT((int32_t)s);
            }
        }
#undef ORC_EMIT
    }
    return e;
}
