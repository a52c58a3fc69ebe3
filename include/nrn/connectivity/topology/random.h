// nrn/connectivity/topology/random.h -- Erdos-Renyi topology
// (reference: include/nrn/connectivity/topology/random.h:8-49).
#pragma once

#include <nrn/connectivity/topology/topology.h>
#include <nrn/core/options.h>

namespace nrn {

struct RandomTopologyOptions {
    NRN_ARG(double, probability, 0.1);
    NRN_ARG(bool, allow_autapses, false);
};

struct RandomTopology {
    RandomTopologyOptions opts;
};

RandomTopology* random_topology_create(const RandomTopologyOptions& opts = {});
void random_topology_destroy(RandomTopology* r);
ConnectivityTensor random_topology_generate(void* self, int64_t n_source, int64_t n_target, int64_t block_size,
                                            torch::Device device);
const RandomTopologyOptions& random_topology_options(const RandomTopology* r);

extern topology_ops random_topology_ops;

inline TopologyGenerator random_topology_as_generator(RandomTopology* r) {
    return TopologyGenerator{static_cast<void*>(r), &random_topology_ops};
}

}  // namespace nrn
