// connectivity.cpp -- ConnectivityTensor, connections and topology generators.
//
// Topology generation keeps the reference's sequence of torch random calls
// (src/connectivity/topology/random.cpp:25-95,
// distance_dependent.cpp:28-144) so that a seeded torch generator yields the
// same connectivity tensors.  connection_deliver runs on the GPU
// (nrn_cuda_block_deliver); the simulation engine instead compiles the
// tensors into a per-synapse CSR once (simulation.cpp).
#include <nrn/connectivity/connect.h>
#include <nrn/connectivity/topology/distance_dependent.h>
#include <nrn/connectivity/topology/random.h>
#include <nrn/network/population.h>
#include <nrn/plasticity/plasticity_rule.h>

#include <algorithm>
#include <cmath>
#include <vector>

#include "support.h"

namespace nrn {

// ------------------------------------------------------------ BlockIndex ----

int64_t BlockIndex::find_block(int64_t target_row, int64_t source_col) const {
    TORCH_CHECK(row_ptr.defined() && col_idx.defined(), "BlockIndex: row_ptr and col_idx must be defined");
    TORCH_CHECK(target_row >= 0 && target_row < n_rows(), "BlockIndex::find_block: target_row out of range");
    auto rp = row_ptr.to(torch::kCPU);
    auto ci = col_idx.to(torch::kCPU);
    const int32_t* r = rp.data_ptr<int32_t>();
    const int32_t* c = ci.data_ptr<int32_t>();
    for (int32_t i = r[target_row]; i < r[target_row + 1]; ++i)
        if (c[i] == static_cast<int32_t>(source_col)) return i;
    return -1;
}

// ---------------------------------------------------- ConnectivityTensor ----

torch::Tensor ConnectivityTensor::effective_weights() const {
    TORCH_CHECK(weights.defined(), "ConnectivityTensor: weights not defined");
    TORCH_CHECK(structural_mask.defined(), "ConnectivityTensor: structural_mask not defined");
    TORCH_CHECK(modulatory_mask.defined(), "ConnectivityTensor: modulatory_mask not defined");
    return weights * structural_mask.to(weights.dtype()) * modulatory_mask.to(weights.dtype());
}

void ConnectivityTensor::to(torch::Device device) {
    for (torch::Tensor* t : {&block_index.row_ptr, &block_index.col_idx, &weights, &structural_mask,
                             &modulatory_mask, &delays})
        if (t->defined()) *t = t->to(device);
    for (auto& kv : synapse_state)
        if (kv.second.defined()) kv.second = kv.second.to(device);
    if (trace_pre && trace_pre->defined()) trace_pre = trace_pre->to(device);
    if (trace_post && trace_post->defined()) trace_post = trace_post->to(device);
}

int64_t ConnectivityTensor::total_capacity() const { return block_index.n_blocks() * block_size * block_size; }

int64_t ConnectivityTensor::active_count() const {
    if (!structural_mask.defined()) return total_capacity();
    return structural_mask.to(torch::kFloat32).sum().item<int64_t>();
}

double ConnectivityTensor::density() const {
    const int64_t cap = total_capacity();
    return cap == 0 ? 0.0 : static_cast<double>(active_count()) / static_cast<double>(cap);
}

// ------------------------------------------------------------ Connection ----

Connection* connection_create(std::shared_ptr<Population> source, std::shared_ptr<Population> target,
                              ConnectivityTensor connectivity, NrnModule synapse, ConnectOptions options) {
    auto* c = new Connection();
    c->source = std::move(source);
    c->target = std::move(target);
    c->connectivity = std::move(connectivity);
    c->synapse = synapse;
    c->options = options;
    return c;
}

void connection_destroy(Connection* conn) { delete conn; }

void connection_deliver(Connection* conn, const torch::Tensor& spikes, double /*t*/, double /*dt*/) {
    auto& ts = conn->target->state;
    if (!state_contains(ts, "I_syn")) return;   // target not initialised yet
    torch::Tensor& I = state_get(ts, "I_syn");
    auto& ct = conn->connectivity;
    const char* w = "connection_deliver";
    TORCH_CHECK(I.is_cuda(), w, ": the target's I_syn must be on a CUDA device");
    torch::Tensor s = spikes.to(I.device(), torch::kFloat32).contiguous();
    TORCH_CHECK(s.numel() == ct.n_source, w, ": spikes must have n_source elements");
    if (ct.weights.device() != I.device()) ct.to(I.device());   // moves once; stays on the GPU
    if (ct.structural_mask.scalar_type() != torch::kFloat32) ct.structural_mask = ct.structural_mask.to(torch::kFloat32);
    if (ct.modulatory_mask.scalar_type() != torch::kFloat32) ct.modulatory_mask = ct.modulatory_mask.to(torch::kFloat32);
    for (torch::Tensor* t : {&ct.block_index.row_ptr, &ct.block_index.col_idx, &ct.weights, &ct.structural_mask,
                             &ct.modulatory_mask})
        if (!t->is_contiguous()) *t = t->contiguous();
    nrn_block_csr_t c{};
    c.row_ptr = ct.block_index.row_ptr.data_ptr<int32_t>();
    c.col_idx = ct.block_index.col_idx.data_ptr<int32_t>();
    c.weights = ct.weights.data_ptr<float>();
    c.structural_mask = ct.structural_mask.data_ptr<float>();
    c.modulatory_mask = ct.modulatory_mask.data_ptr<float>();
    c.block_size = ct.block_size;
    c.n_blocks = ct.block_index.n_blocks();
    c.n_source = ct.n_source;
    c.n_target = ct.n_target;
    float* out = detail::cuda_f32(I, ct.n_target, "I_syn", w);
    detail::check(nrn_cuda_block_deliver(&c, s.data_ptr<float>(), out, detail::stream_of(I)), w);
}

void connection_attach(Connection* conn, PlasticityRule rule) {
    plasticity_initialize(&rule, conn->connectivity);
    conn->plasticity_rules.push_back(rule);
}

void connection_update_plasticity(Connection* conn, const State& pre_state, const State& post_state, double t,
                                  double dt) {
    for (auto& rule : conn->plasticity_rules)
        plasticity_update(&rule, conn->connectivity, pre_state, post_state, t, dt);
}

std::shared_ptr<Connection> connect(std::shared_ptr<Population> source, std::shared_ptr<Population> target,
                                    TopologyGenerator* topology, NrnModule synapse, const ConnectOptions& options) {
    auto ct = topology_generate(topology, source->n, target->n, options.block_size(), torch::kCPU);
    if (options.weight_scale() != 1.0) ct.weights.mul_(options.weight_scale());
    Connection* c = connection_create(std::move(source), std::move(target), std::move(ct), synapse, options);
    return std::shared_ptr<Connection>(c, connection_destroy);
}

// ------------------------------------------------------ Erdos-Renyi ----

topology_ops random_topology_ops = {random_topology_generate};

RandomTopology* random_topology_create(const RandomTopologyOptions& opts) {
    auto* r = new RandomTopology{};
    r->opts = opts;
    return r;
}

void random_topology_destroy(RandomTopology* r) { delete r; }

const RandomTopologyOptions& random_topology_options(const RandomTopology* r) { return r->opts; }

namespace {

ConnectivityTensor block_skeleton(const std::vector<int32_t>& rp, const std::vector<int32_t>& ci, int64_t n_src,
                                  int64_t n_tgt, int64_t B, torch::Device device) {
    ConnectivityTensor ct;
    auto i32 = torch::TensorOptions().dtype(torch::kInt32);
    ct.block_index.row_ptr = torch::from_blob(const_cast<int32_t*>(rp.data()), {static_cast<int64_t>(rp.size())}, i32)
                                 .clone()
                                 .to(device);
    const int64_t nb = static_cast<int64_t>(ci.size());
    ct.block_index.col_idx = nb ? torch::from_blob(const_cast<int32_t*>(ci.data()), {nb}, i32).clone().to(device)
                                : torch::zeros({0}, i32.device(device));
    ct.block_size = B;
    ct.n_source = n_src;
    ct.n_target = n_tgt;
    return ct;
}

}  // namespace

ConnectivityTensor random_topology_generate(void* self, int64_t n_source, int64_t n_target, int64_t block_size,
                                            torch::Device device) {
    auto* r = static_cast<RandomTopology*>(self);
    TORCH_CHECK(block_size > 0, "random_topology_generate: block_size must be > 0");
    const int64_t nsb = (n_source + block_size - 1) / block_size;
    const int64_t ntb = (n_target + block_size - 1) / block_size;
    // every (target block, source block) pair is present
    std::vector<int32_t> rp(ntb + 1), ci(static_cast<size_t>(nsb * ntb));
    for (int64_t row = 0; row <= ntb; ++row) rp[row] = static_cast<int32_t>(row * nsb);
    for (int64_t k = 0; k < nsb * ntb; ++k) ci[k] = static_cast<int32_t>(k % nsb);
    ConnectivityTensor ct = block_skeleton(rp, ci, n_source, n_target, block_size, device);
    const int64_t nb = nsb * ntb;
    auto f32 = torch::TensorOptions().dtype(torch::kFloat32).device(device);
    // the same random draws, in the same order: U[0,1) weights, then the mask
    ct.weights = torch::rand({nb, block_size, block_size}, f32);
    ct.structural_mask = torch::bernoulli(torch::full({nb, block_size, block_size}, r->opts.probability(), f32));
    if (!r->opts.allow_autapses() && n_source == n_target) {
        for (int64_t b = 0; b < std::min(nsb, ntb); ++b) ct.structural_mask[b * nsb + b].diagonal().zero_();
    }
    ct.modulatory_mask = torch::ones({nb, block_size, block_size}, f32);
    ct.delays = torch::ones({nb, block_size, block_size}, torch::TensorOptions().dtype(torch::kInt32).device(device));
    return ct;
}

// ----------------------------------------------- distance-dependent ----

topology_ops distance_dep_topology_ops = {distance_dep_topology_generate};

DistanceDepTopology* distance_dep_topology_create(const DistanceDependentOptions& opts) {
    auto* d = new DistanceDepTopology{};
    d->opts = opts;
    return d;
}

void distance_dep_topology_destroy(DistanceDepTopology* d) { delete d; }

const DistanceDependentOptions& distance_dep_topology_options(const DistanceDepTopology* d) { return d->opts; }

ConnectivityTensor distance_dep_topology_generate(void* self, int64_t n_source, int64_t n_target, int64_t block_size,
                                                  torch::Device device) {
    auto* d = static_cast<DistanceDepTopology*>(self);
    const double sigma = d->opts.sigma(), max_dist = d->opts.max_distance(), min_p = d->opts.min_probability();
    const double two_s2 = 2.0 * sigma * sigma;
    const int64_t B = block_size;
    const int64_t nsb = (n_source + B - 1) / B, ntb = (n_target + B - 1) / B;
    // neurons evenly spaced on [0, max_distance)
    const double ss = n_source > 1 ? max_dist / static_cast<double>(n_source) : 0.0;
    const double ts = n_target > 1 ? max_dist / static_cast<double>(n_target) : 0.0;
    std::vector<int32_t> rp(ntb + 1, 0), ci;
    for (int64_t tr = 0; tr < ntb; ++tr) {
        rp[tr] = static_cast<int32_t>(ci.size());
        const double tc = (tr * B + std::min((tr + 1) * B, n_target)) * 0.5 * ts;
        for (int64_t sc = 0; sc < nsb; ++sc) {
            const double scn = (sc * B + std::min((sc + 1) * B, n_source)) * 0.5 * ss;
            const double dd = std::abs(tc - scn);
            // a block is kept when its centres are close enough to matter
            if (std::exp(-dd * dd / two_s2) > 0.01 || min_p > 0.01) ci.push_back(static_cast<int32_t>(sc));
        }
    }
    rp[ntb] = static_cast<int32_t>(ci.size());
    const int64_t nb = static_cast<int64_t>(ci.size());
    ConnectivityTensor ct = block_skeleton(rp, ci, n_source, n_target, B, device);
    if (nb == 0) ct.block_index.col_idx = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(device));
    auto f32 = torch::TensorOptions().dtype(torch::kFloat32).device(device);
    ct.weights = torch::rand({nb, B, B}, f32);
    ct.structural_mask = torch::zeros({nb, B, B}, f32);
    auto cpu_f32 = torch::TensorOptions().dtype(torch::kFloat32);
    for (int64_t tr = 0; tr < ntb; ++tr) {
        const int64_t t0 = tr * B, t1 = std::min(t0 + B, n_target);
        for (int32_t bi = rp[tr]; bi < rp[tr + 1]; ++bi) {
            const int64_t s0 = static_cast<int64_t>(ci[bi]) * B, s1 = std::min(s0 + B, n_source);
            auto prob = torch::zeros({B, B}, cpu_f32);
            float* pb = prob.data_ptr<float>();
            for (int64_t ti = 0; ti < t1 - t0; ++ti) {
                const double tp = (t0 + ti) * ts;
                for (int64_t si = 0; si < s1 - s0; ++si) {
                    const double dd = std::abs(tp - (s0 + si) * ss);
                    pb[ti * B + si] = static_cast<float>(std::max(std::exp(-dd * dd / two_s2), min_p));
                }
            }
            ct.structural_mask[bi] = torch::bernoulli(prob.to(device));
        }
    }
    ct.modulatory_mask = torch::ones({nb, B, B}, f32);
    ct.delays = torch::ones({nb, B, B}, torch::TensorOptions().dtype(torch::kInt32).device(device));
    return ct;
}

}  // namespace nrn
