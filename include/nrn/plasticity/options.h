// nrn/plasticity/options.h -- pair STDP options (reference: include/nrn/plasticity/options.h:22-30).
#pragma once

#include <nrn/core/options.h>

namespace nrn {

struct STDPOptions {
    NRN_ARG(double, tau_plus, 0.020);
    NRN_ARG(double, tau_minus, 0.020);
    NRN_ARG(double, a_plus, 0.01);
    NRN_ARG(double, a_minus, -0.012);
    NRN_ARG(double, w_max, 1.0);
    NRN_ARG(double, w_min, 0.0);
    NRN_ARG(double, learning_rate, 1.0);
};

}  // namespace nrn
