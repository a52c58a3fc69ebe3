// nrn/simulation/runner.h -- the simulation loop (reference: include/nrn/simulation/runner.h:24-82).
//
// sim_create compiles the Region into a GPU-resident engine (neuron state
// aliased, connectivity as per-synapse CSR); sim_step / sim_run_steps /
// sim_run enqueue steps in CUDA graphs; recorders and callbacks are served
// between graph launches.  Per-synapse delays (ConnectivityTensor::delays)
// are honoured; the reference reads every connection with delay 1
// (src/simulation/runner.cpp:113), which equals this for its generators.
#pragma once

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include <torch/torch.h>

#include <nrn/core/state.h>
#include <nrn/core/types.h>
#include <nrn/monitor/recorder.h>
#include <nrn/network/population.h>
#include <nrn/network/region.h>
#include <nrn/simulation/clock.h>
#include <nrn/simulation/options.h>
#include <nrn/simulation/spike_buffer.h>

namespace nrn {

struct Simulation;
struct SimEngine;   // the GPU engine behind a Simulation (opaque)

using SimCallback = std::function<void(const Simulation&, double)>;

struct Simulation {
    Region* region;
    SimulationOptions options;
    Clock clock;
    std::unordered_map<std::string, SpikeBuffer> spike_buffers;
    std::vector<Recorder> recorders;
    std::vector<std::pair<int64_t, SimCallback>> callbacks;
    std::shared_ptr<SimEngine> engine;
};

Simulation* sim_create(Region* region, SimulationOptions options = {});
void sim_destroy(Simulation* sim);
void sim_record(Simulation* sim, std::shared_ptr<Population> population, std::vector<std::string> variables,
                int64_t subsample = 1);
void sim_run(Simulation* sim);
void sim_run_steps(Simulation* sim, int64_t n);
void sim_step(Simulation* sim);
// Not in the reference: reads back the recorders' pending data and writes
// the plastic weights into the connections' ConnectivityTensors now.
// sim_run / sim_run_steps / sim_destroy do this at their end; a loop of
// sim_step calls leaves both on the device until one of those (or a
// recorder query) runs.
void sim_sync(Simulation* sim);
// [K, 2] float: (neuron id, time)
torch::Tensor sim_get_spikes(const Simulation* sim, const std::shared_ptr<Population>& population);
// [T, N]
torch::Tensor sim_get_recorded(const Simulation* sim, const std::shared_ptr<Population>& population,
                               const std::string& variable);
void sim_add_callback(Simulation* sim, int64_t every_n, SimCallback fn);

}  // namespace nrn
