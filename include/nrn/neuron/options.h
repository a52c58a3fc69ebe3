// nrn/neuron/options.h -- neuron model options, SI units; same fields and
// defaults as the reference (include/nrn/neuron/options.h:23-92).
#pragma once

#include <torch/torch.h>

#include <nrn/core/options.h>

namespace nrn {
namespace neuron {

// Leaky integrate-and-fire.
struct LIFOptions {
    NRN_ARG(double, v_rest, -0.065);     // V
    NRN_ARG(double, v_thresh, -0.050);   // V
    NRN_ARG(double, v_reset, -0.065);    // V
    NRN_ARG(double, tau_m, 0.010);       // s
    NRN_ARG(double, tau_ref, 0.002);     // s
    NRN_ARG(double, c_m, 250e-12);       // F
    NRN_ARG(double, i_bg, 0.0);          // A
    NRN_ARG(torch::Dtype, dtype, torch::kFloat32);
};

// Adaptive exponential integrate-and-fire (Brette & Gerstner 2005).
struct AdExOptions {
    NRN_ARG(double, v_rest, -0.0706);
    NRN_ARG(double, v_thresh, -0.0504);
    NRN_ARG(double, v_reset, -0.0706);
    NRN_ARG(double, v_peak, 0.0);
    NRN_ARG(double, tau_m, 9.37e-3);
    NRN_ARG(double, tau_w, 0.144);
    NRN_ARG(double, tau_ref, 0.002);
    NRN_ARG(double, c_m, 281e-12);
    NRN_ARG(double, g_l, 30e-9);
    NRN_ARG(double, a, 4e-9);
    NRN_ARG(double, b, 80.5e-12);
    NRN_ARG(double, delta_t, 0.002);
    NRN_ARG(double, i_bg, 0.0);
    NRN_ARG(torch::Dtype, dtype, torch::kFloat32);
};

// Izhikevich (2003), dimensionless; dt is converted to milliseconds.
struct IzhikevichOptions {
    NRN_ARG(double, a, 0.02);
    NRN_ARG(double, b, 0.2);
    NRN_ARG(double, c, -65.0);
    NRN_ARG(double, d, 8.0);
    NRN_ARG(double, v_peak, 30.0);
    NRN_ARG(double, v_init, -65.0);
    NRN_ARG(double, u_init, 0.0);   // kept for the API; u starts at b * v_init as in the reference
    NRN_ARG(torch::Dtype, dtype, torch::kFloat32);
};

}  // namespace neuron
}  // namespace nrn
