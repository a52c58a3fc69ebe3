// nrn/plasticity/plasticity_rule.h -- plasticity rule handle
// (reference: include/nrn/plasticity/plasticity_rule.h:19-65).
#pragma once

#include <nrn/core/state.h>
#include <nrn/core/types.h>

namespace nrn {

struct ConnectivityTensor;

struct plasticity_ops {
    void (*initialize)(void* self, ConnectivityTensor& conn);
    void (*update)(void* self, ConnectivityTensor& conn, const State& pre_state, const State& post_state, double t,
                   double dt);
    void (*reset)(void* self);
};

struct PlasticityRule {
    void* impl;
    plasticity_ops* ops;
};

inline void plasticity_initialize(PlasticityRule* r, ConnectivityTensor& conn) { r->ops->initialize(r->impl, conn); }
inline void plasticity_update(PlasticityRule* r, ConnectivityTensor& conn, const State& pre, const State& post,
                              double t, double dt) {
    r->ops->update(r->impl, conn, pre, post, t, dt);
}
inline void plasticity_reset(PlasticityRule* r) { r->ops->reset(r->impl); }

}  // namespace nrn
