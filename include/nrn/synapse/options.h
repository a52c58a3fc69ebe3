// nrn/synapse/options.h -- synapse model options (reference: include/nrn/synapse/options.h).
#pragma once

#include <nrn/core/options.h>

namespace nrn {

struct StaticSynapseOptions {
    NRN_ARG(double, weight, 1.0);
    NRN_ARG(double, delay, 0.001);
};

struct ExponentialSynapseOptions {
    NRN_ARG(double, tau_decay, 0.005);
    NRN_ARG(double, weight, 1.0);
    NRN_ARG(double, delay, 0.001);
};

struct DoubleExponentialSynapseOptions {
    NRN_ARG(double, tau_rise, 0.0005);
    NRN_ARG(double, tau_decay, 0.005);
    NRN_ARG(double, weight, 1.0);
    NRN_ARG(double, delay, 0.001);
};

struct AMPAOptions {
    NRN_ARG(double, tau_rise, 0.0005);
    NRN_ARG(double, tau_decay, 0.005);
    NRN_ARG(double, e_rev, 0.0);
    NRN_ARG(double, weight, 1.0);
    NRN_ARG(double, delay, 0.001);
};

}  // namespace nrn
