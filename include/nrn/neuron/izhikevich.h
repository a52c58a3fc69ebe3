// nrn/neuron/izhikevich.h -- Izhikevich (reference: include/nrn/neuron/izhikevich.h:34-80).
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

struct IzhikevichNeuron {
    int64_t n;
    IzhikevichOptions options;
    // state [N]
    torch::Tensor v;
    torch::Tensor u;
    torch::Tensor spike;
    torch::Tensor I_syn;
    // parameters [N]
    torch::Tensor a;
    torch::Tensor b;
    torch::Tensor c;
    torch::Tensor d;
    torch::Tensor v_peak;
};

IzhikevichNeuron* izh_create(int64_t n, IzhikevichOptions opts = {});
void izh_destroy(IzhikevichNeuron* m);

void izh_forward(void* self, State& state, double t, double dt);
void izh_reset(void* self);
const char** izh_state_vars(void* self, int* count);
int64_t izh_size(void* self);
void izh_to_device(void* self, torch::Device device);

inline void izh_forward(IzhikevichNeuron* m, State& state, double t, double dt) { izh_forward(static_cast<void*>(m), state, t, dt); }
inline void izh_reset(IzhikevichNeuron* m) { izh_reset(static_cast<void*>(m)); }
inline void izh_to_device(IzhikevichNeuron* m, torch::Device device) { izh_to_device(static_cast<void*>(m), device); }

extern nrn_ops izh_ops;

inline NrnModule izh_as_module(IzhikevichNeuron* m) { return NrnModule{static_cast<void*>(m), &izh_ops}; }

}  // namespace neuron
}  // namespace nrn
