// nrn/synapse/double_exponential.h -- rise/decay synapse (reference: include/nrn/synapse/double_exponential.h).
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

struct DoubleExponentialSynapse {
    int64_t n;
    DoubleExponentialSynapseOptions options;
};

DoubleExponentialSynapse* dexp_synapse_create(int64_t n, DoubleExponentialSynapseOptions opts = {});
void dexp_synapse_destroy(DoubleExponentialSynapse* syn);

void dexp_synapse_forward(void* self, State& state, double t, double dt);
void dexp_synapse_reset(void* self);
const char** dexp_synapse_state_vars(void* self, int* count);
int64_t dexp_synapse_size(void* self);
void dexp_synapse_to_device(void* self, torch::Device device);

inline void dexp_synapse_forward(DoubleExponentialSynapse* syn, State& state, double t, double dt) { dexp_synapse_forward(static_cast<void*>(syn), state, t, dt); }
inline void dexp_synapse_reset(DoubleExponentialSynapse* syn) { dexp_synapse_reset(static_cast<void*>(syn)); }
inline void dexp_synapse_to_device(DoubleExponentialSynapse* syn, torch::Device device) { dexp_synapse_to_device(static_cast<void*>(syn), device); }

extern nrn_ops dexp_synapse_ops;

inline NrnModule dexp_synapse_as_module(DoubleExponentialSynapse* syn) { return NrnModule{static_cast<void*>(syn), &dexp_synapse_ops}; }

}  // namespace synapse
}  // namespace nrn
