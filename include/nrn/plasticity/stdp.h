// nrn/plasticity/stdp.h -- pair STDP (reference: include/nrn/plasticity/stdp.h:32-73).
//
// stdp_update on a ConnectivityTensor runs on the GPU over its dense blocks
// with the reference's per-synapse semantics; inside sim_run the engine
// applies the same rule event-driven on its per-synapse CSR.
#pragma once

#include <nrn/plasticity/options.h>
#include <nrn/plasticity/plasticity_rule.h>

namespace nrn {

struct ConnectivityTensor;

struct STDPState {
    STDPOptions opts;
    double cached_dt = 0.0;
    double decay_pre = 0.0;
    double decay_post = 0.0;
};

STDPState* stdp_create(const STDPOptions& opts = {});
void stdp_destroy(STDPState* s);
void stdp_initialize(void* self, ConnectivityTensor& conn);
void stdp_update(void* self, ConnectivityTensor& conn, const State& pre_state, const State& post_state, double t,
                 double dt);
void stdp_reset(void* self);
const STDPOptions& stdp_options(const STDPState* s);

extern plasticity_ops stdp_ops;

inline PlasticityRule stdp_as_rule(STDPState* s) { return PlasticityRule{static_cast<void*>(s), &stdp_ops}; }

}  // namespace nrn
