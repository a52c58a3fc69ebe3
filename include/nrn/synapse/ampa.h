// nrn/synapse/ampa.h -- AMPA receptor synapse (reference: include/nrn/synapse/ampa.h).
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

struct AMPASynapse {
    int64_t n;
    AMPAOptions options;
};

AMPASynapse* ampa_create(int64_t n, AMPAOptions opts = {});
void ampa_destroy(AMPASynapse* syn);

void ampa_forward(void* self, State& state, double t, double dt);
void ampa_reset(void* self);
const char** ampa_state_vars(void* self, int* count);
int64_t ampa_size(void* self);
void ampa_to_device(void* self, torch::Device device);

inline void ampa_forward(AMPASynapse* syn, State& state, double t, double dt) { ampa_forward(static_cast<void*>(syn), state, t, dt); }
inline void ampa_reset(AMPASynapse* syn) { ampa_reset(static_cast<void*>(syn)); }
inline void ampa_to_device(AMPASynapse* syn, torch::Device device) { ampa_to_device(static_cast<void*>(syn), device); }

extern nrn_ops ampa_ops;

inline NrnModule ampa_as_module(AMPASynapse* syn) { return NrnModule{static_cast<void*>(syn), &ampa_ops}; }

}  // namespace synapse
}  // namespace nrn
