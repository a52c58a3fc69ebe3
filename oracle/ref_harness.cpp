// ref_harness.cpp -- drives the reference implementation (synergetics/libnrn,
// compiled unmodified from its own sources into oracle/_ref/libnrn_ref.so)
// on an orc_net description, so that its outputs pin the C restatement
// (nrn_oracle.c) and give the CPU baseline.
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile into oracle/_ref/.
//
// What runs is the reference's own code:
//   neuron updates      nrn_forward -> lif/adex/izh_forward (CPU torch path)
//   delivery            connection_deliver            (src/connectivity/connect.cpp:36-79)
//   delay lines         SpikeBuffer::push / read       (src/simulation/spike_buffer.cpp)
//   plasticity          connection_update_plasticity -> stdp_update (src/plasticity/stdp.cpp)
//   clock, set-up       sim_create, Clock              (src/simulation/runner.cpp:17-42)
// The step loop restates sim_step's phases (runner.cpp:95-173) because the
// reference's own loop reads only delay 1 (runner.cpp:113) and has no
// external drive.  The extensions, identical to nrn_oracle.c:
//   * per-synapse delays: each projection is split into one Connection per
//     (delay, multapse layer), delivered from spike_buffers.read(delay);
//   * external drive from Philox (oracle_common.h), added to I_syn after P2;
//   * conductance input for AdEx (oracle_common.h orc_cond_current), added
//     to I_syn before the reference's forward.
#include <chrono>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include <torch/torch.h>

#include <nrn/connectivity/connect.h>
#include <nrn/connectivity/topology/random.h>
#include <nrn/network/population.h>
#include <nrn/network/region.h>
#include <nrn/neuron/adex.h>
#include <nrn/neuron/izhikevich.h>
#include <nrn/neuron/lif.h>
#include <nrn/plasticity/stdp.h>
#include <nrn/simulation/runner.h>
#include <nrn/synapse/static.h>

#include "oracle_common.h"

using namespace nrn;

namespace {

torch::Tensor from_f32(const float* p, int64_t n) {
    return torch::from_blob(const_cast<float*>(p), {n}, torch::kFloat32).clone();
}

struct Group {
    Connection* conn;
    int proj;
    int delay;
    std::vector<std::tuple<int64_t, int64_t, int, int>> where;  // (k, block, row, col)
};

// Builds a block-CSR ConnectivityTensor (only non-empty blocks) holding the
// synapses `ks` of projection Q; each (target, source) pair appears once.
ConnectivityTensor make_ct(const orc_proj& Q, const std::vector<int64_t>& ks,
                           int64_t n_src, int64_t n_tgt, int64_t B, Group& g) {
    int64_t ntb = (n_tgt + B - 1) / B, nsb = (n_src + B - 1) / B;
    std::map<std::pair<int64_t, int64_t>, int64_t> blocks;   // (tb, sb) -> idx
    for (int64_t k : ks) blocks[{Q.tgt[k] / B, Q.src[k] / B}] = 0;
    int64_t nb = 0;
    std::vector<int32_t> rp(ntb + 1, 0), ci;
    for (auto& kv : blocks) { kv.second = nb++; rp[kv.first.first + 1]++; ci.push_back((int32_t)kv.first.second); }
    for (int64_t r = 0; r < ntb; ++r) rp[r + 1] += rp[r];
    (void)nsb;
    ConnectivityTensor ct;
    ct.block_index.row_ptr = torch::from_blob(rp.data(), {ntb + 1}, torch::kInt32).clone();
    ct.block_index.col_idx = torch::from_blob(ci.data(), {nb}, torch::kInt32).clone();
    ct.block_size = B;
    ct.n_source = n_src;
    ct.n_target = n_tgt;
    ct.weights = torch::zeros({nb, B, B}, torch::kFloat32);
    ct.structural_mask = torch::zeros({nb, B, B}, torch::kFloat32);
    ct.modulatory_mask = torch::ones({nb, B, B}, torch::kFloat32);
    ct.delays = torch::ones({nb, B, B}, torch::kInt32);
    float* W = ct.weights.data_ptr<float>();
    float* M = ct.structural_mask.data_ptr<float>();
    int32_t* D = ct.delays.data_ptr<int32_t>();
    for (int64_t k : ks) {
        int64_t b = blocks[{Q.tgt[k] / B, Q.src[k] / B}];
        int r = (int)(Q.tgt[k] % B), c = (int)(Q.src[k] % B);
        size_t o = ((size_t)b * B + r) * B + c;
        W[o] = Q.w[k];
        M[o] = 1.0f;
        D[o] = Q.delay[k];
        g.where.emplace_back(k, b, r, c);
    }
    return ct;
}

NrnModule make_module(const orc_pop& P, void** raw) {
    int64_t n = P.n;
    auto hp = [&](int k) { return from_f32(P.hp + (size_t)k * n, n); };
    if (P.model == ORC_LIF) {
        auto o = neuron::LIFOptions().v_rest(P.p[0]).v_thresh(P.p[1]).v_reset(P.p[2])
                     .tau_m(P.p[3]).tau_ref(P.p[4]).c_m(P.p[5]).i_bg(P.p[6]);
        auto* m = neuron::lif_create(n, o);
        if (P.hp) {
            m->v_rest = hp(0); m->v_thresh = hp(1); m->v_reset = hp(2); m->tau_m = hp(3);
            m->tau_ref = hp(4); m->c_m = hp(5); m->i_bg = hp(6);
        }
        if (P.init_v) m->v = from_f32(P.init_v, n);
        *raw = m;
        return neuron::lif_as_module(m);
    }
    if (P.model == ORC_ADEX) {
        auto o = neuron::AdExOptions().v_rest(P.p[0]).v_thresh(P.p[1]).v_reset(P.p[2])
                     .v_peak(P.p[3]).tau_m(P.p[4]).tau_w(P.p[5]).tau_ref(P.p[6]).c_m(P.p[7])
                     .g_l(P.p[8]).a(P.p[9]).b(P.p[10]).delta_t(P.p[11]).i_bg(P.p[12]);
        auto* m = neuron::adex_create(n, o);
        if (P.hp) {
            m->v_rest = hp(0); m->v_thresh = hp(1); m->v_reset = hp(2); m->v_peak = hp(3);
            m->tau_m = hp(4); m->tau_w = hp(5); m->tau_ref = hp(6); m->c_m = hp(7);
            m->g_l = hp(8); m->a = hp(9); m->b = hp(10); m->delta_t = hp(11); m->i_bg = hp(12);
        }
        if (P.init_v) m->v = from_f32(P.init_v, n);
        if (P.init_aux) m->w = from_f32(P.init_aux, n);
        *raw = m;
        return neuron::adex_as_module(m);
    }
    auto o = neuron::IzhikevichOptions().a(P.p[0]).b(P.p[1]).c(P.p[2]).d(P.p[3]).v_peak(P.p[4]);
    auto* m = neuron::izh_create(n, o);
    if (P.hp) { m->a = hp(0); m->b = hp(1); m->c = hp(2); m->d = hp(3); m->v_peak = hp(4); }
    if (P.init_v) m->v = from_f32(P.init_v, n);
    if (P.init_aux) m->u = from_f32(P.init_aux, n);
    *raw = m;
    return neuron::izh_as_module(m);
}

void destroy_module(const orc_pop& P, void* raw) {
    if (P.model == ORC_LIF) neuron::lif_destroy(static_cast<neuron::LIFNeuron*>(raw));
    else if (P.model == ORC_ADEX) neuron::adex_destroy(static_cast<neuron::AdExNeuron*>(raw));
    else neuron::izh_destroy(static_cast<neuron::IzhikevichNeuron*>(raw));
}

}  // namespace

extern "C" {

// Runs the network through the reference.  Returns 0 (1 when spike_cap was
// too small); *elapsed_s receives the wall time of the step loop alone.
__attribute__((visibility("default")))
int ref_net_run(const orc_net* net, int64_t block_size, double* elapsed_s) {
    if (net->threads > 0) torch::set_num_threads(net->threads);
    int np = net->npop, nq = net->nproj;
    int maxd = 1;
    for (int q = 0; q < nq; ++q)
        for (int64_t k = 0; k < net->projs[q].nnz; ++k)
            maxd = std::max(maxd, (int)net->projs[q].delay[k]);

    auto* region = region_create("oracle");
    std::vector<std::shared_ptr<Population>> pops(np), gexc(np), ginh(np);
    std::vector<void*> raws(np);
    auto* syn = synapse::static_synapse_create(1);
    auto synm = synapse::static_synapse_as_module(syn);
    std::vector<char> cond(np, 0);
    for (int q = 0; q < nq; ++q)
        if (net->projs[q].receptor != ORC_RECV_CURRENT) cond[net->projs[q].tgt_pop] = 1;
    for (int p = 0; p < np; ++p) {
        const orc_pop& P = net->pops[p];
        if (P.drive_kind == ORC_DRIVE_POISSON_GEXC) cond[p] = 1;
        auto mod = make_module(P, &raws[p]);
        pops[p] = std::shared_ptr<Population>(
            population_create("pop" + std::to_string(p), mod, P.n, torch::kCPU), population_destroy);
        region_add_population(region, pops[p]);
        // Proxy populations whose "I_syn" collects conductance input.
        for (int r = 0; r < 2; ++r) {
            auto* px = population_create("g" + std::to_string(r) + "_" + std::to_string(p), mod, P.n,
                                         torch::kCPU);
            px->state["I_syn"] = torch::zeros({P.n}, torch::kFloat32);
            (r == 0 ? gexc : ginh)[p] = std::shared_ptr<Population>(px, population_destroy);
        }
    }
    auto sopts = SimulationOptions().dt_fast(net->dt).dt_slow(net->dt * std::max(1, net->slow_ratio))
                     .dt_structural(net->dt * std::max(1, net->slow_ratio)).max_delay_steps(maxd + 1)
                     .device(torch::kCPU);
    Simulation* sim = sim_create(region, sopts);   // runs forward(dt = 0) once

    // Connections: one per (projection, delay, multapse layer).
    std::vector<Group> groups;
    std::vector<STDPState*> stdps;
    for (int q = 0; q < nq; ++q) {
        const orc_proj& Q = net->projs[q];
        std::map<std::pair<int, int>, std::vector<int64_t>> parts;   // (delay, layer)
        std::map<std::tuple<int, int32_t, int32_t>, int> seen;       // (delay, tgt, src) -> count
        for (int64_t k = 0; k < Q.nnz; ++k) {
            int layer = seen[{Q.delay[k], Q.tgt[k], Q.src[k]}]++;
            parts[{Q.delay[k], layer}].push_back(k);
        }
        auto tgt = Q.receptor == ORC_RECV_CURRENT ? pops[Q.tgt_pop]
                 : Q.receptor == ORC_RECV_GEXC ? gexc[Q.tgt_pop] : ginh[Q.tgt_pop];
        for (auto& kv : parts) {
            Group g;
            g.proj = q;
            g.delay = kv.first.first;
            auto ct = make_ct(Q, kv.second, net->pops[Q.src_pop].n, net->pops[Q.tgt_pop].n,
                              block_size, g);
            g.conn = connection_create(pops[Q.src_pop], tgt, std::move(ct), synm,
                                       ConnectOptions().block_size(block_size));
            if (Q.plastic) {
                auto* s = stdp_create(STDPOptions().tau_plus(Q.stdp[0]).tau_minus(Q.stdp[1])
                                          .a_plus(Q.stdp[2]).a_minus(Q.stdp[3]).w_min(Q.stdp[4])
                                          .w_max(Q.stdp[5]).learning_rate(Q.stdp[6]));
                stdps.push_back(s);
                connection_attach(g.conn, stdp_as_rule(s));
            }
            groups.push_back(std::move(g));
        }
    }

    int64_t N = 0;
    for (int p = 0; p < np; ++p) N += net->pops[p].n;
    int64_t nspk = 0;
    auto t0 = std::chrono::steady_clock::now();
    for (int t = 0; t < net->steps; ++t) {
        double time = sim->clock.time();
        double dt = net->dt;
        // P1
        for (int p = 0; p < np; ++p) {
            state_get(pops[p]->state, "I_syn").zero_();
            gexc[p]->state["I_syn"].zero_();
            ginh[p]->state["I_syn"].zero_();
        }
        // P2
        for (auto& g : groups) {
            auto spikes = sim->spike_buffers.at(g.conn->source->name).read(g.delay);
            connection_deliver(g.conn, spikes, time, dt);
        }
        // drive and conductance input
        for (int p = 0; p < np; ++p) {
            const orc_pop& P = net->pops[p];
            float* I = state_get(pops[p]->state, "I_syn").data_ptr<float>();
            float* ge = gexc[p]->state["I_syn"].data_ptr<float>();
            if (P.drive_kind != ORC_DRIVE_NONE) {
                float d0 = (float)P.drive[0], d1 = (float)P.drive[1];
                float en = (float)std::exp(-P.drive[0]);
                float* dst = P.drive_kind == ORC_DRIVE_POISSON_GEXC ? ge : I;
                for (int i = 0; i < P.n; ++i) {
                    uint32_t gid = (uint32_t)(P.offset + i);
                    dst[i] += orc_drive_value(P.drive_kind, d0, d1, en, net->seed, gid, (uint32_t)t);
                }
            }
            if (cond[p]) {
                // Conductance state lives in the proxies' "g" entries.
                auto& gs = gexc[p]->state;
                if (!gs.count("g")) { gs["g"] = torch::zeros({P.n}); ginh[p]->state["g"] = torch::zeros({P.n}); }
                float* gE = gs["g"].data_ptr<float>();
                float* gI = ginh[p]->state["g"].data_ptr<float>();
                const float* gi_in = ginh[p]->state["I_syn"].data_ptr<float>();
                const float* v = state_get(pops[p]->state, "v").data_ptr<float>();
                float de = (float)std::exp(-dt / P.cond[0]), di = (float)std::exp(-dt / P.cond[1]);
                for (int i = 0; i < P.n; ++i)
                    I[i] = orc_cond_current(I[i], &gE[i], &gI[i], ge[i], gi_in[i], de, di,
                                            (float)P.cond[2], (float)P.cond[3], v[i]);
            }
        }
        // P3
        for (int p = 0; p < np; ++p) nrn_forward(&pops[p]->module, pops[p]->state, time, dt);
        // P4
        for (int p = 0; p < np; ++p)
            sim->spike_buffers.at(pops[p]->name).push(state_get(pops[p]->state, "spike"));
        // P5
        if (sim->clock.is_slow_boundary()) {
            for (auto& g : groups)
                if (!g.conn->plasticity_rules.empty())
                    connection_update_plasticity(g.conn, g.conn->source->state,
                                                 pops[net->projs[g.proj].tgt_pop]->state, time, dt);
        }
        // P6
        for (int p = 0; p < np; ++p) {
            const float* s = state_get(pops[p]->state, "spike").data_ptr<float>();
            for (int i = 0; i < net->pops[p].n; ++i) {
                if (s[i] != 0.0f) {
                    if (nspk < net->spike_cap) {
                        net->spike_step[nspk] = t;
                        net->spike_id[nspk] = net->pops[p].offset + i;
                    }
                    ++nspk;
                }
            }
        }
        if (net->trace_n > 0 && net->trace_v) {
            for (int k = 0; k < net->trace_n; ++k) {
                int g = net->trace_ids[k], p = 0;
                while (p + 1 < np && net->pops[p + 1].offset <= g) ++p;
                net->trace_v[(size_t)t * net->trace_n + k] =
                    state_get(pops[p]->state, "v").data_ptr<float>()[g - net->pops[p].offset];
            }
        }
        sim->clock.advance_fast();
    }
    auto t1 = std::chrono::steady_clock::now();
    if (elapsed_s) *elapsed_s = std::chrono::duration<double>(t1 - t0).count();
    if (net->n_spikes) *net->n_spikes = nspk;

    for (int p = 0; p < np; ++p) {
        const orc_pop& P = net->pops[p];
        auto& st = pops[p]->state;
        if (net->final_v) std::memcpy(net->final_v + P.offset, st["v"].data_ptr<float>(), P.n * 4);
        if (net->final_aux) {
            const char* key = P.model == ORC_ADEX ? "w" : P.model == ORC_IZH ? "u" : nullptr;
            if (key) std::memcpy(net->final_aux + P.offset, st[key].data_ptr<float>(), P.n * 4);
            else std::memset(net->final_aux + P.offset, 0, P.n * 4);
        }
        if (net->final_ref) {
            if (st.count("refractory"))
                std::memcpy(net->final_ref + P.offset, st["refractory"].data_ptr<float>(), P.n * 4);
            else std::memset(net->final_ref + P.offset, 0, P.n * 4);
        }
    }
    for (auto& g : groups) {
        float* out = net->projs[g.proj].w_out;
        if (out) {
            const float* W = g.conn->connectivity.weights.data_ptr<float>();
            int64_t B = g.conn->connectivity.block_size;
            for (auto& [k, b, r, c] : g.where) out[k] = W[((size_t)b * B + r) * B + c];
        }
        connection_destroy(g.conn);
    }
    for (auto* s : stdps) stdp_destroy(s);
    sim_destroy(sim);
    region_destroy(region);
    for (int p = 0; p < np; ++p) {
        pops[p].reset(); gexc[p].reset(); ginh[p].reset();
        destroy_module(net->pops[p], raws[p]);
    }
    synapse::static_synapse_destroy(syn);
    return nspk > net->spike_cap ? 1 : 0;
}

// Neuron-only run: the reference's *_forward called directly with the given
// per-step input current, as tests/neuron/test_neuron_dynamics.cpp does.
__attribute__((visibility("default")))
int ref_neuron_run(const orc_pop* P, int steps, double dt, const float* I,
                   float* out_v, float* out_aux, float* out_ref, uint8_t* out_spike) {
    void* raw = nullptr;
    NrnModule m = make_module(*P, &raw);
    State state;
    int64_t n = P->n;
    for (int t = 0; t < steps; ++t) {
        torch::Tensor Isyn;
        if (P->model == ORC_LIF) Isyn = static_cast<neuron::LIFNeuron*>(raw)->I_syn;
        else if (P->model == ORC_ADEX) Isyn = static_cast<neuron::AdExNeuron*>(raw)->I_syn;
        else Isyn = static_cast<neuron::IzhikevichNeuron*>(raw)->I_syn;
        if (I) std::memcpy(Isyn.data_ptr<float>(), I + (size_t)t * n, n * 4);
        nrn_forward(&m, state, t * dt, dt);
        size_t o = (size_t)t * n;
        if (out_v) std::memcpy(out_v + o, state["v"].data_ptr<float>(), n * 4);
        if (out_aux) {
            const char* key = P->model == ORC_ADEX ? "w" : P->model == ORC_IZH ? "u" : nullptr;
            if (key) std::memcpy(out_aux + o, state[key].data_ptr<float>(), n * 4);
        }
        if (out_ref && state.count("refractory"))
            std::memcpy(out_ref + o, state["refractory"].data_ptr<float>(), n * 4);
        if (out_spike) {
            const float* s = state["spike"].data_ptr<float>();
            for (int64_t i = 0; i < n; ++i) out_spike[o + i] = s[i] != 0.0f;
        }
    }
    destroy_module(*P, raw);
    return 0;
}

// The reference's Erdos-Renyi connect() after torch::manual_seed(seed):
// exports the block CSR, weights and structural mask (each [n_blocks,B,B]).
__attribute__((visibility("default")))
int64_t ref_er_connect(int64_t n_src, int64_t n_tgt, int64_t B, double p, int autapses,
                       double weight_scale, uint64_t seed, int same_population,
                       int32_t* row_ptr, int32_t* col_idx, float* weights, float* mask,
                       int64_t cap_blocks) {
    torch::manual_seed(seed);
    auto* topo = random_topology_create(RandomTopologyOptions().probability(p).allow_autapses(autapses != 0));
    auto gen = random_topology_as_generator(topo);
    auto* lif = neuron::lif_create(std::max(n_src, n_tgt));
    auto mod = neuron::lif_as_module(lif);
    auto src = std::shared_ptr<Population>(population_create("s", mod, n_src, torch::kCPU), population_destroy);
    std::shared_ptr<Population> tgt = same_population ? src
        : std::shared_ptr<Population>(population_create("t", mod, n_tgt, torch::kCPU), population_destroy);
    auto* syn = synapse::static_synapse_create(1);
    auto conn = connect(src, tgt, &gen, synapse::static_synapse_as_module(syn),
                        ConnectOptions().block_size(B).weight_scale(weight_scale));
    auto& ct = conn->connectivity;
    int64_t nb = ct.block_index.n_blocks();
    if (nb <= cap_blocks) {
        std::memcpy(row_ptr, ct.block_index.row_ptr.data_ptr<int32_t>(), (ct.block_index.n_rows() + 1) * 4);
        std::memcpy(col_idx, ct.block_index.col_idx.data_ptr<int32_t>(), nb * 4);
        std::memcpy(weights, ct.weights.contiguous().data_ptr<float>(), nb * B * B * 4);
        std::memcpy(mask, ct.structural_mask.contiguous().data_ptr<float>(), nb * B * B * 4);
    }
    conn.reset();
    synapse::static_synapse_destroy(syn);
    random_topology_destroy(topo);
    neuron::lif_destroy(lif);
    return nb;
}

}  // extern "C"
