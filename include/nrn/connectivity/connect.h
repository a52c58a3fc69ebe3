// nrn/connectivity/connect.h -- connections between populations
// (reference: include/nrn/connectivity/connect.h:24-68).
#pragma once

#include <memory>
#include <vector>

#include <torch/torch.h>

#include <nrn/connectivity/connectivity_tensor.h>
#include <nrn/connectivity/options.h>
#include <nrn/core/module.h>
#include <nrn/core/state.h>
#include <nrn/core/types.h>

namespace nrn {

struct Population;
struct PlasticityRule;
struct TopologyGenerator;

struct Connection {
    std::shared_ptr<Population> source;
    std::shared_ptr<Population> target;
    ConnectivityTensor connectivity;
    NrnModule synapse;
    ConnectOptions options;
    std::vector<PlasticityRule> plasticity_rules;
};

Connection* connection_create(std::shared_ptr<Population> source, std::shared_ptr<Population> target,
                              ConnectivityTensor connectivity, NrnModule synapse, ConnectOptions options);
void connection_destroy(Connection* conn);

// I_syn(target) += (W * M_s * M_m) . spikes, on the GPU.
void connection_deliver(Connection* conn, const torch::Tensor& spikes, double t, double dt);

void connection_attach(Connection* conn, PlasticityRule rule);
void connection_update_plasticity(Connection* conn, const State& pre_state, const State& post_state, double t,
                                  double dt);

std::shared_ptr<Connection> connect(std::shared_ptr<Population> source, std::shared_ptr<Population> target,
                                    TopologyGenerator* topology, NrnModule synapse,
                                    const ConnectOptions& options = {});

}  // namespace nrn
