// plasticity.cpp -- pair STDP rule of the nrn:: API.
//
// stdp_update (src/plasticity/stdp.cpp:43-141) runs on the GPU over the
// connection's dense blocks (nrn_cuda_block_stdp) with per-synapse traces,
// the reference's operation order and its clamp of every in-range entry.
// Inside sim_run the engine applies the same rule event by event on its
// per-synapse CSR and writes the weights back afterwards.
#include <nrn/connectivity/connectivity_tensor.h>
#include <nrn/plasticity/stdp.h>

#include <cmath>

#include "support.h"

namespace nrn {

plasticity_ops stdp_ops = {stdp_initialize, stdp_update, stdp_reset};

STDPState* stdp_create(const STDPOptions& opts) {
    auto* s = new STDPState{};
    s->opts = opts;
    return s;
}

void stdp_destroy(STDPState* s) { delete s; }

void stdp_initialize(void* /*self*/, ConnectivityTensor& conn) {
    TORCH_CHECK(conn.weights.defined(), "stdp_initialize: weights tensor must be defined");
    conn.trace_pre = torch::zeros_like(conn.weights);
    conn.trace_post = torch::zeros_like(conn.weights);
}

void stdp_update(void* self, ConnectivityTensor& conn, const State& pre_state, const State& post_state,
                 double /*t*/, double dt) {
    auto* s = static_cast<STDPState*>(self);
    if (dt != s->cached_dt) {
        s->cached_dt = dt;
        s->decay_pre = std::exp(-dt / s->opts.tau_plus());
        s->decay_post = std::exp(-dt / s->opts.tau_minus());
    }
    if (!state_contains(pre_state, "spike") || !state_contains(post_state, "spike")) return;
    if (!conn.trace_pre.has_value() || !conn.trace_post.has_value()) return;
    const char* w = "stdp_update";
    const torch::Tensor& pre = state_get(pre_state, "spike");
    const torch::Tensor& post = state_get(post_state, "spike");
    TORCH_CHECK(pre.is_cuda() && post.is_cuda(), w, ": spike tensors must be on a CUDA device");
    if (conn.weights.device() != pre.device()) conn.to(pre.device());
    auto pre_c = pre.to(torch::kFloat32).contiguous();
    auto post_c = post.to(torch::kFloat32).contiguous();
    TORCH_CHECK(pre_c.numel() == conn.n_source && post_c.numel() == conn.n_target, w, ": spike sizes");
    for (torch::Tensor* t : {&conn.structural_mask, &conn.modulatory_mask})
        if (t->scalar_type() != torch::kFloat32) *t = t->to(torch::kFloat32);
    for (torch::Tensor* t : {&conn.block_index.row_ptr, &conn.block_index.col_idx, &conn.weights,
                             &conn.structural_mask, &conn.modulatory_mask, &*conn.trace_pre, &*conn.trace_post})
        if (!t->is_contiguous()) *t = t->contiguous();
    nrn_block_csr_t c{};
    c.row_ptr = conn.block_index.row_ptr.data_ptr<int32_t>();
    c.col_idx = conn.block_index.col_idx.data_ptr<int32_t>();
    c.weights = conn.weights.data_ptr<float>();
    c.structural_mask = conn.structural_mask.data_ptr<float>();
    c.modulatory_mask = conn.modulatory_mask.data_ptr<float>();
    c.block_size = conn.block_size;
    c.n_blocks = conn.block_index.n_blocks();
    c.n_source = conn.n_source;
    c.n_target = conn.n_target;
    const float params[7] = {static_cast<float>(s->decay_pre), static_cast<float>(s->decay_post),
                             static_cast<float>(s->opts.a_plus()), static_cast<float>(std::abs(s->opts.a_minus())),
                             static_cast<float>(s->opts.learning_rate()), static_cast<float>(s->opts.w_min()),
                             static_cast<float>(s->opts.w_max())};
    detail::check(nrn_cuda_block_stdp(&c, conn.weights.data_ptr<float>(), conn.trace_pre->data_ptr<float>(),
                                      conn.trace_post->data_ptr<float>(), pre_c.data_ptr<float>(),
                                      post_c.data_ptr<float>(), params, detail::stream_of(pre_c)),
                  w);
}

void stdp_reset(void* self) {
    auto* s = static_cast<STDPState*>(self);
    s->cached_dt = 0.0;
    s->decay_pre = 0.0;
    s->decay_post = 0.0;
}

const STDPOptions& stdp_options(const STDPState* s) { return s->opts; }

}  // namespace nrn
