// nrn/connectivity/topology/distance_dependent.h -- Gaussian distance-dependent
// topology (reference: include/nrn/connectivity/topology/distance_dependent.h:9-58).
#pragma once

#include <nrn/connectivity/topology/topology.h>
#include <nrn/core/options.h>

namespace nrn {

struct DistanceDependentOptions {
    NRN_ARG(double, sigma, 200.0e-6);
    NRN_ARG(double, max_distance, 1000.0e-6);
    NRN_ARG(double, min_probability, 0.0);
};

struct DistanceDepTopology {
    DistanceDependentOptions opts;
};

DistanceDepTopology* distance_dep_topology_create(const DistanceDependentOptions& opts = {});
void distance_dep_topology_destroy(DistanceDepTopology* d);
ConnectivityTensor distance_dep_topology_generate(void* self, int64_t n_source, int64_t n_target,
                                                  int64_t block_size, torch::Device device);
const DistanceDependentOptions& distance_dep_topology_options(const DistanceDepTopology* d);

extern topology_ops distance_dep_topology_ops;

inline TopologyGenerator distance_dep_topology_as_generator(DistanceDepTopology* d) {
    return TopologyGenerator{static_cast<void*>(d), &distance_dep_topology_ops};
}

}  // namespace nrn
