// nrn/simulation/options.h -- simulation options (reference: include/nrn/simulation/options.h:11-19).
#pragma once

#include <torch/torch.h>

#include <nrn/core/options.h>
#include <nrn/core/types.h>

namespace nrn {

struct SimulationOptions {
    NRN_ARG(Duration, dt_fast, 0.0001);
    NRN_ARG(Duration, dt_slow, 0.01);
    NRN_ARG(Duration, dt_structural, 1.0);
    NRN_ARG(Duration, duration, 1.0);
    NRN_ARG(torch::Device, device, torch::kCUDA);
    NRN_ARG(bool, use_cuda_graphs, true);   // steps run in captured CUDA graphs
    NRN_ARG(int64_t, max_delay_steps, 50);
};

}  // namespace nrn
