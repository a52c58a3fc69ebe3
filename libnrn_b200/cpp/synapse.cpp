// synapse.cpp -- synapse modules of the nrn:: API.
//
// A Connection carries one of these handles (Connection::synapse); the
// reference never calls their forward from its step loop
// (src/synapse/static.cpp:37-42 is a no-op, the others throw,
// src/synapse/exponential.cpp:37-42).  The same behaviour is kept here.
// Conductance synapses for the simulation are part of the engine (AdEx
// populations with g_exc/g_inh input, include/nrn_cuda.h).
#include <nrn/synapse/synapse.h>

#include "support.h"

namespace nrn {
namespace synapse {

namespace {
const char* kISyn[] = {"I_syn"};
const char* kAmpa[] = {"I_syn", "g", "s_rise", "s_decay"};
}  // namespace

#define NRN_SYNAPSE_IMPL(Type, prefix, Opts, nvars, vars, forward_body)                    \
    Type* prefix##_create(int64_t n, Opts opts) {                                       \
        TORCH_CHECK(n >= 0, #prefix "_create: n must be >= 0");                         \
        auto* s = new Type();                                                            \
        s->n = n;                                                                        \
        s->options = opts;                                                               \
        return s;                                                                        \
    }                                                                                    \
    void prefix##_destroy(Type* s) { delete s; }                                         \
    void prefix##_forward(void*, State&, double, double) { forward_body; }               \
    void prefix##_reset(void*) {}                                                        \
    const char** prefix##_state_vars(void*, int* count) {                                \
        *count = nvars;                                                                  \
        return vars;                                                                     \
    }                                                                                    \
    int64_t prefix##_size(void* self) { return static_cast<Type*>(self)->n; }           \
    void prefix##_to_device(void*, torch::Device) {}                                     \
    nrn_ops prefix##_ops = {prefix##_forward, prefix##_reset, prefix##_state_vars, prefix##_size, \
                            prefix##_to_device};

NRN_SYNAPSE_IMPL(StaticSynapse, static_synapse, StaticSynapseOptions, 1, kISyn, (void)0)
NRN_SYNAPSE_IMPL(ExponentialSynapse, exp_synapse, ExponentialSynapseOptions, 1, kISyn,
                 TORCH_CHECK(false, "exp_synapse_forward: synapses act through connection_deliver "
                                    "(not implemented as a module, as in the reference)"))
NRN_SYNAPSE_IMPL(DoubleExponentialSynapse, dexp_synapse, DoubleExponentialSynapseOptions, 1, kISyn,
                 TORCH_CHECK(false, "dexp_synapse_forward: synapses act through connection_deliver "
                                    "(not implemented as a module, as in the reference)"))
NRN_SYNAPSE_IMPL(AMPASynapse, ampa, AMPAOptions, 4, kAmpa,
                 TORCH_CHECK(false, "ampa_forward: synapses act through connection_deliver "
                                    "(not implemented as a module, as in the reference)"))

#undef NRN_SYNAPSE_IMPL

}  // namespace synapse
}  // namespace nrn
