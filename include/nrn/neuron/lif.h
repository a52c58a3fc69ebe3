// nrn/neuron/lif.h -- leaky integrate-and-fire (reference: include/nrn/neuron/lif.h:34-82).
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

struct LIFNeuron {
    int64_t n;
    LIFOptions options;
    // state [N]
    torch::Tensor v;
    torch::Tensor spike;
    torch::Tensor refractory;
    torch::Tensor I_syn;
    // parameters [N] (per-neuron heterogeneity)
    torch::Tensor v_rest;
    torch::Tensor v_thresh;
    torch::Tensor v_reset;
    torch::Tensor tau_m;
    torch::Tensor tau_ref;
    torch::Tensor c_m;
    torch::Tensor i_bg;
};

LIFNeuron* lif_create(int64_t n, LIFOptions opts = {});
void lif_destroy(LIFNeuron* m);

void lif_forward(void* self, State& state, double t, double dt);
void lif_reset(void* self);
const char** lif_state_vars(void* self, int* count);
int64_t lif_size(void* self);
void lif_to_device(void* self, torch::Device device);

inline void lif_forward(LIFNeuron* m, State& state, double t, double dt) { lif_forward(static_cast<void*>(m), state, t, dt); }
inline void lif_reset(LIFNeuron* m) { lif_reset(static_cast<void*>(m)); }
inline void lif_to_device(LIFNeuron* m, torch::Device device) { lif_to_device(static_cast<void*>(m), device); }

extern nrn_ops lif_ops;

inline NrnModule lif_as_module(LIFNeuron* m) { return NrnModule{static_cast<void*>(m), &lif_ops}; }

}  // namespace neuron
}  // namespace nrn
