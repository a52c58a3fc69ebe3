// api_bench -- the Brunel network of the reference's example configuration
// (10,000 E + 2,500 I LIF, connection probability 0.1, so in-degree about
// 1,000 + 250, dt 0.1 ms, pair STDP on E->E; the random topology gives every
// synapse a delay of one step, as the reference's does) built and run
// only through the nrn:: C++ API, as a user program of the reference would.
// It times the same number of steps twice on the GPU engine behind the API:
// one sim_run_steps(N) call, and N sim_step calls; each measurement ends
// with sim_sync (spikes read back, weights written into the
// ConnectivityTensor) and a device synchronisation.  Prints one JSON line.
//
//   api_bench [steps]
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <memory>
#include <string>

#include <cuda_runtime.h>
#include <torch/torch.h>

#include <nrn/nrn.h>

using namespace nrn;
using namespace nrn::literals;

namespace {

struct Net {
    Region* region = nullptr;
    Simulation* sim = nullptr;
    std::shared_ptr<Population> exc, inh;
    int64_t nnz = 0;
};

Net build(int64_t ne, int64_t ni) {
    Net n;
    const torch::Device dev(torch::kCUDA);
    torch::manual_seed(1);
    auto o = neuron::LIFOptions().v_rest(0.0_mV).v_thresh(20.0_mV).v_reset(10.0_mV).tau_m(20.0_ms).tau_ref(2.0_ms)
                 .c_m(250.0_pF).i_bg(270.0_pA);
    auto* el = neuron::lif_create(ne, o);
    auto* il = neuron::lif_create(ni, o);
    neuron::lif_to_device(el, dev);
    neuron::lif_to_device(il, dev);
    el->v.copy_(0.020 * torch::rand({ne}, torch::TensorOptions().device(dev)));
    il->v.copy_(0.020 * torch::rand({ni}, torch::TensorOptions().device(dev)));
    n.exc = std::shared_ptr<Population>(population_create("exc", neuron::lif_as_module(el), ne, dev), population_destroy);
    n.inh = std::shared_ptr<Population>(population_create("inh", neuron::lif_as_module(il), ni, dev), population_destroy);
    auto* topo = random_topology_create(RandomTopologyOptions().probability(0.1));
    auto gen = random_topology_as_generator(topo);
    auto* syn = synapse::static_synapse_create(1);
    auto sm = synapse::static_synapse_as_module(syn);
    const double je = 0.1e-3 * 250e-12 / 1e-4 * 2.0, ji = -5.0 * je;   // mean weight J c_m / dt
    auto opt = [](double w) { return ConnectOptions().block_size(256).weight_scale(w); };
    auto ee = connect(n.exc, n.exc, &gen, sm, opt(je));
    auto ei = connect(n.exc, n.inh, &gen, sm, opt(je));
    auto ie = connect(n.inh, n.exc, &gen, sm, opt(ji));
    auto ii = connect(n.inh, n.inh, &gen, sm, opt(ji));
    random_topology_destroy(topo);
    auto* stdp = stdp_create(STDPOptions().tau_plus(20.0_ms).tau_minus(20.0_ms).a_plus(0.01).a_minus(-0.0105)
                                 .learning_rate(je).w_min(0.0).w_max(2.0 * je));
    connection_attach(ee.get(), stdp_as_rule(stdp));
    n.region = region_create("brunel");
    region_add_population(n.region, n.exc);
    region_add_population(n.region, n.inh);
    for (auto& c : {ee, ei, ie, ii}) {
        region_add_connection(n.region, c);
        n.nnz += (c->connectivity.structural_mask != 0).sum().item<int64_t>();
    }
    n.sim = sim_create(n.region, SimulationOptions().dt_fast(0.1_ms).dt_slow(0.1_ms).dt_structural(10.0_ms)
                                     .duration(1.0_s).max_delay_steps(32).device(dev));
    sim_record(n.sim, n.exc, {"spike"});
    sim_record(n.sim, n.inh, {"spike"});
    return n;
}

double timed(const std::function<void()>& f) {
    cudaDeviceSynchronize();
    const auto t0 = std::chrono::steady_clock::now();
    f();
    cudaDeviceSynchronize();
    return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

}  // namespace

int main(int argc, char** argv) {
    const int64_t steps = argc > 1 ? std::atoll(argv[1]) : 2000;
    Net n = build(10'000, 2'500);
    sim_run_steps(n.sim, 200);   // warm-up: engine build, graph capture
    sim_sync(n.sim);
    for (int k = 0; k < 20; ++k) sim_step(n.sim);
    sim_sync(n.sim);
    const int64_t s0 = sim_get_spikes(n.sim, n.exc).size(0) + sim_get_spikes(n.sim, n.inh).size(0);
    const double t_run = timed([&] {
        sim_run_steps(n.sim, steps);
        sim_sync(n.sim);
    });
    const int64_t s1 = sim_get_spikes(n.sim, n.exc).size(0) + sim_get_spikes(n.sim, n.inh).size(0);
    double t_host = 0.0;   // the loop's own time, before the final sim_sync
    const double t_step = timed([&] {
        const auto t0 = std::chrono::steady_clock::now();
        for (int64_t k = 0; k < steps; ++k) sim_step(n.sim);
        t_host = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        sim_sync(n.sim);
    });
    const int64_t s2 = sim_get_spikes(n.sim, n.exc).size(0) + sim_get_spikes(n.sim, n.inh).size(0);
    const double mean_out = static_cast<double>(n.nnz) / 12'500.0;
    const double dt = 1e-4;
    std::printf(
        "{\"metric\": \"synaptic_events_per_s\", \"path\": \"nrn:: C++ API (libnrn.so)\", \"workload\": "
        "\"Brunel 10,000 E + 2,500 I, p = 0.1, delay 1 step, STDP on E->E\", \"steps\": %lld, \"synapses\": %lld, "
        "\"sim_run_steps\": {\"ms_per_step\": %.5f, \"rtf\": %.4f, \"events_per_s\": %.4e, \"spikes\": %lld}, "
        "\"sim_step_loop\": {\"ms_per_step\": %.5f, \"host_ms_per_step\": %.5f, \"rtf\": %.4f, \"events_per_s\": %.4e, "
        "\"spikes\": %lld}, "
        "\"step_over_run\": %.3f}\n",
        static_cast<long long>(steps), static_cast<long long>(n.nnz), t_run / steps * 1e3, t_run / (steps * dt),
        (s1 - s0) * mean_out / t_run, static_cast<long long>(s1 - s0), t_step / steps * 1e3, t_host / steps * 1e3,
        t_step / (steps * dt),
        (s2 - s1) * mean_out / t_step, static_cast<long long>(s2 - s1), t_step / t_run);
    sim_destroy(n.sim);
    region_destroy(n.region);
    return 0;
}
