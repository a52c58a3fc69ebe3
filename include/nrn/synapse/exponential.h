// nrn/synapse/exponential.h -- single-exponential synapse (reference: include/nrn/synapse/exponential.h).
//
// Synapse modules are handles a Connection carries (Connection::synapse);
// the step loop never calls their forward -- delivery goes through the
// connectivity (connection_deliver / the engine), as in the reference.
#pragma once

#include <torch/torch.h>

#include <nrn/core/module.h>
#include <nrn/core/state.h>
#include <nrn/core/types.h>
#include <nrn/synapse/options.h>

namespace nrn {
namespace synapse {

struct ExponentialSynapse {
    int64_t n;
    ExponentialSynapseOptions options;
};

ExponentialSynapse* exp_synapse_create(int64_t n, ExponentialSynapseOptions opts = {});
void exp_synapse_destroy(ExponentialSynapse* syn);

void exp_synapse_forward(void* self, State& state, double t, double dt);
void exp_synapse_reset(void* self);
const char** exp_synapse_state_vars(void* self, int* count);
int64_t exp_synapse_size(void* self);
void exp_synapse_to_device(void* self, torch::Device device);

inline void exp_synapse_forward(ExponentialSynapse* syn, State& state, double t, double dt) { exp_synapse_forward(static_cast<void*>(syn), state, t, dt); }
inline void exp_synapse_reset(ExponentialSynapse* syn) { exp_synapse_reset(static_cast<void*>(syn)); }
inline void exp_synapse_to_device(ExponentialSynapse* syn, torch::Device device) { exp_synapse_to_device(static_cast<void*>(syn), device); }

extern nrn_ops exp_synapse_ops;

inline NrnModule exp_synapse_as_module(ExponentialSynapse* syn) { return NrnModule{static_cast<void*>(syn), &exp_synapse_ops}; }

}  // namespace synapse
}  // namespace nrn
