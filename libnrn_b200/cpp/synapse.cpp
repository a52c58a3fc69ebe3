// synapse.cpp -- synapse modules of the nrn:: API.
//
// The reference declares these models (include/nrn/synapse/exponential.h:16-21,
// double_exponential.h:17-25, ampa.h:17-29) but its forwards are stubs
// (src/synapse/exponential.cpp:37-42 throws; static.cpp is a no-op).  Here
// they act in two places:
//   * in a simulation, a Connection whose synapse module is one of these
//     delivers into a synapse channel of its target population, whose state
//     the fused neuron update advances on the device (include/nrn_cuda.h,
//     nrn_syn_desc_t; the mapping is in simulation.cpp);
//   * called directly, forward advances the module's state variables in the
//     given State by one step of dt with the same equations, spikes having
//     been added by connection_deliver beforehand:
//       exponential:   I_syn <- I_syn * exp(-dt/tau_decay)
//       double exp.:   I_rise, I_decay decay with their time constants,
//                      I_syn = I_decay - I_rise
//       AMPA:          s_rise, s_decay decay, g = weight * (s_decay - s_rise),
//                      I_syn = g * (v - e_rev) when the State holds "v"
//     (the declared sign: I_syn is the outward membrane current).
//   Decay factors are (float)exp(-dt/tau), as in the engine.
#include <nrn/synapse/synapse.h>

#include <cmath>

#include "support.h"

namespace nrn {
namespace synapse {

namespace {
const char* kISyn[] = {"I_syn"};
const char* kDexp[] = {"I_syn", "I_rise", "I_decay"};
const char* kAmpa[] = {"I_syn", "g", "s_rise", "s_decay"};

float decay(double dt, double tau) {
    TORCH_CHECK(tau > 0.0, "synapse time constants must be positive");
    return static_cast<float>(std::exp(-dt / tau));
}

void scale_(State& s, const char* name, float f) {
    auto& t = state_get(s, name);
    t.mul_(f);
}
}  // namespace

#define NRN_SYNAPSE_IMPL(Type, prefix, Opts, nvars, vars)                                 \
    Type* prefix##_create(int64_t n, Opts opts) {                                       \
        TORCH_CHECK(n >= 0, #prefix "_create: n must be >= 0");                         \
        auto* s = new Type();                                                            \
        s->n = n;                                                                        \
        s->options = opts;                                                               \
        return s;                                                                        \
    }                                                                                    \
    void prefix##_destroy(Type* s) { delete s; }                                         \
    void prefix##_reset(void*) {}                                                        \
    const char** prefix##_state_vars(void*, int* count) {                                \
        *count = nvars;                                                                  \
        return vars;                                                                     \
    }                                                                                    \
    int64_t prefix##_size(void* self) { return static_cast<Type*>(self)->n; }           \
    void prefix##_to_device(void*, torch::Device) {}                                     \
    nrn_ops prefix##_ops = {prefix##_forward, prefix##_reset, prefix##_state_vars, prefix##_size, \
                            prefix##_to_device};

// A static synapse has no dynamics of its own (its weight is the delivered
// current), as in the reference.
void static_synapse_forward(void*, State&, double, double) {}

void exp_synapse_forward(void* self, State& s, double, double dt) {
    const auto& o = static_cast<ExponentialSynapse*>(self)->options;
    scale_(s, "I_syn", decay(dt, o.tau_decay()));
}

void dexp_synapse_forward(void* self, State& s, double, double dt) {
    const auto& o = static_cast<DoubleExponentialSynapse*>(self)->options;
    scale_(s, "I_rise", decay(dt, o.tau_rise()));
    scale_(s, "I_decay", decay(dt, o.tau_decay()));
    state_get(s, "I_syn").copy_(state_get(s, "I_decay") - state_get(s, "I_rise"));
}

void ampa_forward(void* self, State& s, double, double dt) {
    const auto& o = static_cast<AMPASynapse*>(self)->options;
    scale_(s, "s_rise", decay(dt, o.tau_rise()));
    scale_(s, "s_decay", decay(dt, o.tau_decay()));
    auto& g = state_get(s, "g");
    g.copy_((state_get(s, "s_decay") - state_get(s, "s_rise")) * static_cast<float>(o.weight()));
    if (state_contains(s, "v")) state_get(s, "I_syn").copy_(g * (state_get(s, "v") - static_cast<float>(o.e_rev())));
}

NRN_SYNAPSE_IMPL(StaticSynapse, static_synapse, StaticSynapseOptions, 1, kISyn)
NRN_SYNAPSE_IMPL(ExponentialSynapse, exp_synapse, ExponentialSynapseOptions, 1, kISyn)
NRN_SYNAPSE_IMPL(DoubleExponentialSynapse, dexp_synapse, DoubleExponentialSynapseOptions, 3, kDexp)
NRN_SYNAPSE_IMPL(AMPASynapse, ampa, AMPAOptions, 4, kAmpa)

#undef NRN_SYNAPSE_IMPL

}  // namespace synapse
}  // namespace nrn
