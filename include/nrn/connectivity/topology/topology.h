// nrn/connectivity/topology/topology.h -- topology generator handle
// (reference: include/nrn/connectivity/topology/topology.h:23-55).
#pragma once

#include <torch/torch.h>

#include <nrn/connectivity/connectivity_tensor.h>

namespace nrn {

struct topology_ops {
    ConnectivityTensor (*generate)(void* self, int64_t n_source, int64_t n_target, int64_t block_size,
                                   torch::Device device);
};

struct TopologyGenerator {
    void* impl;
    topology_ops* ops;
};

inline ConnectivityTensor topology_generate(TopologyGenerator* g, int64_t n_src, int64_t n_tgt, int64_t block_size,
                                            torch::Device device) {
    return g->ops->generate(g->impl, n_src, n_tgt, block_size, device);
}

}  // namespace nrn
