// A user program written only against the nrn:: API.  The same source is
// compiled against the reference (oracle/Makefile: run on the CPU, its
// working path) and against this library (run on the GPU); the two outputs
// are compared by tests/test_cpp_api.py.
//
//   dropin_brunel <out.bin> <cpu|cuda> [steps]
// Writes: int32 n_exc_spikes, n_inh_spikes, n_w, then the spikes as
// (float id, float time) pairs (exc then inh), then the E->E weights.
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <string>
#include <vector>

#include <torch/torch.h>

#include <nrn/connectivity/connect.h>
#include <nrn/connectivity/topology/random.h>
#include <nrn/core/types.h>
#include <nrn/network/population.h>
#include <nrn/network/region.h>
#include <nrn/neuron/lif.h>
#include <nrn/plasticity/stdp.h>
#include <nrn/simulation/options.h>
#include <nrn/simulation/runner.h>
#include <nrn/synapse/static.h>

using namespace nrn;
using namespace nrn::literals;

int main(int argc, char** argv) {
    if (argc < 3) return 2;
    const torch::Device device = std::string(argv[2]) == "cuda" ? torch::Device(torch::kCUDA) : torch::Device(torch::kCPU);
    const int steps = argc > 3 ? std::atoi(argv[3]) : 300;
    torch::manual_seed(2024);
    const int64_t ne = 400, ni = 100;
    auto eo = neuron::LIFOptions().v_rest(-65.0_mV).v_thresh(-50.0_mV).v_reset(-65.0_mV).tau_m(20.0_ms)
                  .tau_ref(2.0_ms).c_m(250.0_pF).i_bg(300.0_pA);
    auto* el = neuron::lif_create(ne, eo);
    auto* il = neuron::lif_create(ni, eo.tau_m(10.0_ms).i_bg(400.0_pA));
    neuron::lif_to_device(el, device);
    neuron::lif_to_device(il, device);
    // initial potentials U(-65, -50) mV, drawn on the CPU from the seeded generator
    el->v.copy_(-0.065 + 0.015 * torch::rand({ne}));
    il->v.copy_(-0.065 + 0.015 * torch::rand({ni}));
    auto exc = std::shared_ptr<Population>(population_create("exc", neuron::lif_as_module(el), ne, device),
                                           population_destroy);
    auto inh = std::shared_ptr<Population>(population_create("inh", neuron::lif_as_module(il), ni, device),
                                           population_destroy);
    auto* topo = random_topology_create(RandomTopologyOptions().probability(0.1));
    auto gen = random_topology_as_generator(topo);
    auto* syn = synapse::static_synapse_create(1);
    auto sm = synapse::static_synapse_as_module(syn);
    const double je = 250.0e-12, ji = -5.0 * je;
    auto ee = connect(exc, exc, &gen, sm, ConnectOptions().block_size(64).weight_scale(je));
    auto ei = connect(exc, inh, &gen, sm, ConnectOptions().block_size(64).weight_scale(je));
    auto ie = connect(inh, exc, &gen, sm, ConnectOptions().block_size(64).weight_scale(ji));
    auto ii = connect(inh, inh, &gen, sm, ConnectOptions().block_size(64).weight_scale(ji));
    auto* stdp = stdp_create(STDPOptions().tau_plus(20.0_ms).tau_minus(20.0_ms).a_plus(0.01).a_minus(-0.012)
                                 .learning_rate(1e-9).w_min(0.0).w_max(je * 2));
    connection_attach(ee.get(), stdp_as_rule(stdp));
    auto* region = region_create("dropin");
    region_add_population(region, exc);
    region_add_population(region, inh);
    for (auto& c : {ee, ei, ie, ii}) region_add_connection(region, c);
    auto* sim = sim_create(region, SimulationOptions().dt_fast(0.1_ms).dt_slow(1.0_ms).dt_structural(10.0_ms)
                                       .device(device));
    sim_record(sim, exc, {"spike"});
    sim_record(sim, inh, {"spike"});
    sim_run_steps(sim, steps);
    auto se = sim_get_spikes(sim, exc).contiguous();
    auto si = sim_get_spikes(sim, inh).contiguous();
    auto w = ee->connectivity.weights.to(torch::kCPU).contiguous();
    FILE* f = std::fopen(argv[1], "wb");
    if (!f) return 3;
    int32_t hdr[3] = {static_cast<int32_t>(se.size(0)), static_cast<int32_t>(si.size(0)),
                      static_cast<int32_t>(w.numel())};
    std::fwrite(hdr, 4, 3, f);
    std::fwrite(se.data_ptr<float>(), 4, se.numel(), f);
    std::fwrite(si.data_ptr<float>(), 4, si.numel(), f);
    std::fwrite(w.data_ptr<float>(), 4, w.numel(), f);
    std::fclose(f);
    std::printf("exc spikes %d inh spikes %d\n", hdr[0], hdr[1]);
    sim_destroy(sim);
    region_destroy(region);
    ee.reset(); ei.reset(); ie.reset(); ii.reset();
    exc.reset(); inh.reset();
    stdp_destroy(stdp);
    synapse::static_synapse_destroy(syn);
    random_topology_destroy(topo);
    neuron::lif_destroy(el);
    neuron::lif_destroy(il);
    return 0;
}
