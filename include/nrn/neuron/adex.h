// nrn/neuron/adex.h -- adaptive exponential integrate-and-fire (reference: include/nrn/neuron/adex.h:35-90).
//
// State and parameter tensors live on the GPU (float32, [N]); *_forward runs
// one fused CUDA update (nrn_cuda_pop_step) on the current CUDA stream and
// publishes the state tensors into the State map.  There is no CPU path:
// forward on CPU tensors raises c10::Error.
#pragma once

#include <torch/torch.h>

#include <nrn/core/module.h>
#include <nrn/core/state.h>
#include <nrn/core/types.h>
#include <nrn/neuron/options.h>

namespace nrn {
namespace neuron {

struct AdExNeuron {
    int64_t n;
    AdExOptions options;
    // state [N]
    torch::Tensor v;
    torch::Tensor w;
    torch::Tensor spike;
    torch::Tensor refractory;
    torch::Tensor I_syn;
    // parameters [N]
    torch::Tensor v_rest;
    torch::Tensor v_thresh;
    torch::Tensor v_reset;
    torch::Tensor v_peak;
    torch::Tensor tau_m;
    torch::Tensor tau_w;
    torch::Tensor tau_ref;
    torch::Tensor c_m;
    torch::Tensor g_l;
    torch::Tensor a;
    torch::Tensor b;
    torch::Tensor delta_t;
    torch::Tensor i_bg;
};

AdExNeuron* adex_create(int64_t n, AdExOptions opts = {});
void adex_destroy(AdExNeuron* m);

void adex_forward(void* self, State& state, double t, double dt);
void adex_reset(void* self);
const char** adex_state_vars(void* self, int* count);
int64_t adex_size(void* self);
void adex_to_device(void* self, torch::Device device);

inline void adex_forward(AdExNeuron* m, State& state, double t, double dt) { adex_forward(static_cast<void*>(m), state, t, dt); }
inline void adex_reset(AdExNeuron* m) { adex_reset(static_cast<void*>(m)); }
inline void adex_to_device(AdExNeuron* m, torch::Device device) { adex_to_device(static_cast<void*>(m), device); }

extern nrn_ops adex_ops;

inline NrnModule adex_as_module(AdExNeuron* m) { return NrnModule{static_cast<void*>(m), &adex_ops}; }

}  // namespace neuron
}  // namespace nrn
