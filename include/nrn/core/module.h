// nrn/core/module.h -- type-erased module handle and its operations table
// (reference: include/nrn/core/module.h:20-61).
#pragma once

#include <cstdint>
#include <string>

#include <torch/torch.h>

#include <nrn/core/state.h>
#include <nrn/core/types.h>

namespace nrn {

struct nrn_ops {
    void (*forward)(void* self, State& state, double t, double dt);
    void (*reset)(void* self);
    const char** (*state_vars)(void* self, int* count);
    int64_t (*size)(void* self);
    void (*to_device)(void* self, torch::Device device);
};

struct NrnModule {
    void* impl;       // concrete model (LIFNeuron*, AdExNeuron*, ...)
    nrn_ops* ops;     // its operations
};

inline void nrn_forward(NrnModule* m, State& state, double t, double dt) { m->ops->forward(m->impl, state, t, dt); }
inline void nrn_reset(NrnModule* m) { m->ops->reset(m->impl); }
inline int64_t nrn_size(NrnModule* m) { return m->ops->size(m->impl); }
inline void nrn_to_device(NrnModule* m, torch::Device device) { m->ops->to_device(m->impl, device); }
inline const char** nrn_state_vars(NrnModule* m, int* count) { return m->ops->state_vars(m->impl, count); }

}  // namespace nrn
