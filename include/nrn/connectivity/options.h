// nrn/connectivity/options.h -- connection options (reference: include/nrn/connectivity/options.h:11-30).
#pragma once

#include <torch/torch.h>

#include <nrn/core/options.h>

namespace nrn {

enum class ConnectivityRepresentation {
    BlockDense,   // block-dense weights with mask overlays (the API's storage)
    Sparse,
    Procedural,
};

inline constexpr auto BlockDense = ConnectivityRepresentation::BlockDense;
inline constexpr auto Sparse = ConnectivityRepresentation::Sparse;
inline constexpr auto Procedural = ConnectivityRepresentation::Procedural;

struct ConnectOptions {
    NRN_ARG(int64_t, block_size, 256);
    NRN_ARG(ConnectivityRepresentation, representation, BlockDense);
    NRN_ARG(double, weight_scale, 1.0);
    NRN_ARG(bool, with_delays, true);
    NRN_ARG(double, default_delay, 0.001);
    NRN_ARG(torch::Dtype, weight_dtype, torch::kFloat32);
    NRN_ARG(torch::Dtype, mask_dtype, torch::kFloat16);
};

}  // namespace nrn
