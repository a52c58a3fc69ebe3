// The reference's behavioural suites re-expressed against this library's
// nrn:: API (tests/neuron/test_neuron_dynamics.cpp, tests/neuron/test_lif.cpp,
// test_adex.cpp, test_izhikevich.cpp, tests/plasticity/test_stdp.cpp,
// tests/integration/test_brunel_network.cpp).  Needs a CUDA GPU.
#include <nrn/nrn.h>
#include <nrn/config/config.h>

#include <unistd.h>

#include <cstdio>

#include "nrn_test.h"

using namespace nrn;

TEST(LIF, ConstructionOnGpu) {
    auto* lif = neuron::lif_create(10);
    EXPECT_TRUE(lif->v.is_cuda());
    EXPECT_EQ(lif->v.size(0), 10);
    EXPECT_NEAR(lif->v[0].item<float>(), -0.065, 1e-7);
    int count = 0;
    neuron::lif_state_vars(lif, &count);
    EXPECT_EQ(count, 4);
    EXPECT_EQ(neuron::lif_size(lif), 10);
    neuron::lif_destroy(lif);
}

TEST(LIFDynamics, ConstantCurrentProducesSpikes) {
    auto opts = neuron::LIFOptions().v_rest(-0.065).v_thresh(-0.050).v_reset(-0.065).tau_m(0.010).tau_ref(0.002)
                    .c_m(250e-12).i_bg(0.0);
    auto* lif = neuron::lif_create(1, opts);
    lif->I_syn.fill_(500e-12);
    State state;
    int spikes = 0;
    for (int step = 0; step < 1000; ++step) {
        neuron::lif_forward(lif, state, step * 1e-4, 1e-4);
        if (state_get(state, "spike")[0].item<float>() > 0.5f) ++spikes;
        lif->I_syn.fill_(500e-12);
    }
    EXPECT_GT(spikes, 5);
    EXPECT_LT(spikes, 200);
    neuron::lif_destroy(lif);
}

TEST(LIFDynamics, SubthresholdCurrentNoSpikes) {
    auto* lif = neuron::lif_create(1);
    lif->I_syn.fill_(100e-12);
    State state;
    int spikes = 0;
    for (int step = 0; step < 1000; ++step) {
        neuron::lif_forward(lif, state, step * 1e-4, 1e-4);
        spikes += state_get(state, "spike")[0].item<float>() > 0.5f;
        lif->I_syn.fill_(100e-12);
    }
    EXPECT_EQ(spikes, 0);
    neuron::lif_destroy(lif);
}

TEST(LIFDynamics, VoltageRelaxesToRest) {
    auto* lif = neuron::lif_create(1);
    lif->v.fill_(-0.055);
    State state;
    for (int step = 0; step < 2000; ++step) neuron::lif_forward(lif, state, step * 1e-4, 1e-4);
    EXPECT_NEAR(state_get(state, "v")[0].item<float>(), -0.065, 1e-5);
    neuron::lif_destroy(lif);
}

TEST(LIFDynamics, RefractoryPeriodBlocks) {
    auto* lif = neuron::lif_create(1, neuron::LIFOptions().tau_ref(0.005));
    State state;
    lif->v.fill_(-0.049);
    neuron::lif_forward(lif, state, 0.0, 1e-4);
    EXPECT_GT(state_get(state, "spike")[0].item<float>(), 0.5f);
    int next = -1;
    for (int step = 1; step < 200; ++step) {
        lif->I_syn.fill_(500e-12);
        neuron::lif_forward(lif, state, step * 1e-4, 1e-4);
        if (state_get(state, "spike")[0].item<float>() > 0.5f) {
            next = step;
            break;
        }
    }
    EXPECT_GT(next, 45);
    neuron::lif_destroy(lif);
}

TEST(LIFDynamics, MultipleNeuronsIndependent) {
    auto* lif = neuron::lif_create(100);
    auto I = torch::zeros({100});
    I.slice(0, 0, 50).fill_(500e-12);
    State state;
    int first = 0, second = 0;
    for (int step = 0; step < 500; ++step) {
        lif->I_syn.copy_(I);
        neuron::lif_forward(lif, state, step * 1e-4, 1e-4);
        auto s = state_get(state, "spike");
        first += s.slice(0, 0, 50).sum().item<int>();
        second += s.slice(0, 50, 100).sum().item<int>();
    }
    EXPECT_GT(first, 0);
    EXPECT_EQ(second, 0);
    neuron::lif_destroy(lif);
}

TEST(AdExDynamics, SpikesAndAdaptation) {
    auto* adex = neuron::adex_create(1);
    State state;
    int spikes = 0;
    for (int step = 0; step < 2000; ++step) {
        adex->I_syn.fill_(1e-9);
        neuron::adex_forward(adex, state, step * 1e-4, 1e-4);
        spikes += state_get(state, "spike")[0].item<float>() > 0.5f;
    }
    EXPECT_GT(spikes, 1);
    EXPECT_GT(state_get(state, "w")[0].item<float>(), 0.0f);
    neuron::adex_destroy(adex);
}

TEST(IzhikevichDynamics, InputAndNoInput) {
    auto* izh = neuron::izh_create(2);
    State state;
    int s0 = 0, s1 = 0;
    for (int step = 0; step < 1000; ++step) {
        izh->I_syn[0] = 10.0;
        neuron::izh_forward(izh, state, step * 1e-3, 1e-3);
        auto s = state_get(state, "spike");
        s0 += s[0].item<float>() > 0.5f;
        s1 += s[1].item<float>() > 0.5f;
    }
    EXPECT_GT(s0, 5);
    EXPECT_EQ(s1, 0);
    EXPECT_NEAR(neuron::izh_create(1)->u[0].item<float>(), 0.2 * -65.0, 1e-5);
    neuron::izh_destroy(izh);
}

TEST(NoCpuPath, ForwardOnCpuThrows) {
    auto* lif = neuron::lif_create(4);
    neuron::lif_to_device(lif, torch::kCPU);
    State state;
    EXPECT_THROW(neuron::lif_forward(lif, state, 0.0, 1e-4), c10::Error);
    neuron::lif_destroy(lif);
}

TEST(ConnectionDeliver, ProducesNonzeroISyn) {
    auto* lif = neuron::lif_create(32);
    auto pop = std::shared_ptr<Population>(population_create("neurons", neuron::lif_as_module(lif), 32, torch::kCUDA),
                                           population_destroy);
    auto* topo = random_topology_create(RandomTopologyOptions().probability(0.5));
    auto gen = random_topology_as_generator(topo);
    auto* syn = synapse::static_synapse_create(1);
    auto conn = connect(pop, pop, &gen, synapse::static_synapse_as_module(syn), ConnectOptions().block_size(16));
    State state;
    neuron::lif_forward(lif, state, 0.0, 0.0);
    pop->state = state;
    auto spikes = torch::zeros({32});
    spikes[0] = 1.0;
    connection_deliver(conn.get(), spikes, 0.0, 1e-4);
    auto I = state_get(pop->state, "I_syn");
    EXPECT_GT(I.abs().sum().item<float>(), 0.0f);
    // I_syn equals the effective weights' column of source 0: blocks (r, 0)
    auto W = conn->connectivity.effective_weights().to(torch::kCPU);
    auto Ih = I.to(torch::kCPU);
    for (int t = 0; t < 32; ++t)
        EXPECT_NEAR(Ih[t].item<float>(), W[(t / 16) * 2][t % 16][0].item<float>(), 1e-30);
    random_topology_destroy(topo);
    synapse::static_synapse_destroy(syn);
    neuron::lif_destroy(lif);
}

TEST(STDP, InitializeAndUpdateChangesWeights) {
    ConnectivityTensor ct;
    ct.block_index.row_ptr = torch::tensor({0, 1}, torch::kInt32);
    ct.block_index.col_idx = torch::tensor({0}, torch::kInt32);
    ct.block_size = 4;
    ct.n_source = 4;
    ct.n_target = 4;
    ct.weights = torch::full({1, 4, 4}, 0.5);
    ct.structural_mask = torch::ones({1, 4, 4});
    ct.modulatory_mask = torch::ones({1, 4, 4});
    ct.delays = torch::ones({1, 4, 4}, torch::kInt32);
    auto* s = stdp_create(STDPOptions().w_max(1.0).w_min(0.0));
    stdp_initialize(s, ct);
    EXPECT_TRUE(ct.trace_pre.has_value() && ct.trace_post.has_value());
    EXPECT_TRUE(torch::all(*ct.trace_pre == 0).item<bool>());
    State pre, post;
    pre["spike"] = torch::tensor({1.f, 0.f, 0.f, 0.f}, torch::kCUDA);
    post["spike"] = torch::tensor({0.f, 1.f, 0.f, 0.f}, torch::kCUDA);
    stdp_update(s, ct, pre, post, 0.0, 1e-4);
    auto W = ct.weights.to(torch::kCPU);
    // target 1 spiked with source 0: dw = a_plus*1*1 - a_minus*1*1 = 0.01 - 0.012
    EXPECT_NEAR(W[0][1][0].item<float>(), 0.5 + (0.01 - 0.012), 1e-6);
    // source 0 spiked, target 0 silent: dw = -a_minus * 0 (no post trace) = 0
    EXPECT_NEAR(W[0][0][0].item<float>(), 0.5, 1e-7);
    // target 1 spiked, source 1 silent: dw = a_plus * 0 = 0
    EXPECT_NEAR(W[0][1][1].item<float>(), 0.5, 1e-7);
    stdp_destroy(s);
}

namespace {

struct Brunel {
    std::vector<neuron::LIFNeuron*> lifs;
    std::shared_ptr<Population> exc, inh;
    std::vector<std::shared_ptr<Connection>> conns;
    Region* region = nullptr;
    RandomTopology* topo = nullptr;
    synapse::StaticSynapse* syn = nullptr;
    STDPState* stdp = nullptr;

    Brunel(int ne, int ni, double g, bool with_stdp) {
        torch::manual_seed(42);
        auto eo = neuron::LIFOptions().v_rest(-0.065).v_thresh(-0.050).v_reset(-0.065).tau_m(0.020).tau_ref(0.002)
                      .c_m(250e-12).i_bg(400e-12);
        lifs = {neuron::lif_create(ne, eo), neuron::lif_create(ni, eo.tau_m(0.010))};
        for (auto* l : lifs) l->v.copy_(-0.065 + 0.015 * torch::rand({l->n}));
        exc = std::shared_ptr<Population>(population_create("exc", neuron::lif_as_module(lifs[0]), ne, torch::kCUDA),
                                          population_destroy);
        inh = std::shared_ptr<Population>(population_create("inh", neuron::lif_as_module(lifs[1]), ni, torch::kCUDA),
                                          population_destroy);
        topo = random_topology_create(RandomTopologyOptions().probability(0.1));
        auto gen = random_topology_as_generator(topo);
        syn = synapse::static_synapse_create(1);
        auto sm = synapse::static_synapse_as_module(syn);
        const double je = 500e-12, ji = -g * 500e-12;
        conns.push_back(connect(exc, exc, &gen, sm, ConnectOptions().block_size(64).weight_scale(je)));
        conns.push_back(connect(exc, inh, &gen, sm, ConnectOptions().block_size(64).weight_scale(je)));
        conns.push_back(connect(inh, exc, &gen, sm, ConnectOptions().block_size(64).weight_scale(ji)));
        conns.push_back(connect(inh, inh, &gen, sm, ConnectOptions().block_size(64).weight_scale(ji)));
        if (with_stdp) {
            stdp = stdp_create(STDPOptions().learning_rate(1e-3).w_min(0.0).w_max(je * 5));
            connection_attach(conns[0].get(), stdp_as_rule(stdp));
        }
        region = region_create("brunel");
        region_add_population(region, exc);
        region_add_population(region, inh);
        for (auto& c : conns) region_add_connection(region, c);
    }
    ~Brunel() {
        region_destroy(region);
        conns.clear();
        exc.reset();
        inh.reset();
        for (auto* l : lifs) neuron::lif_destroy(l);
        random_topology_destroy(topo);
        synapse::static_synapse_destroy(syn);
        if (stdp) stdp_destroy(stdp);
    }
};

}  // namespace

TEST(BrunelNetwork, RatesInRange) {
    Brunel b(200, 50, 5.0, false);
    auto* sim = sim_create(b.region, SimulationOptions().dt_fast(1e-4).dt_slow(1e-2).dt_structural(1.0).duration(0.1));
    sim_record(sim, b.exc, {"spike"});
    sim_record(sim, b.inh, {"spike"});
    sim_run(sim);
    const double re = sim_get_spikes(sim, b.exc).size(0) / (200 * 0.1);
    const double ri = sim_get_spikes(sim, b.inh).size(0) / (50 * 0.1);
    EXPECT_GT(re, 0.0);
    EXPECT_LT(re, 200.0);
    EXPECT_GT(ri, 0.0);
    EXPECT_LT(ri, 200.0);
    EXPECT_EQ(sim->clock.step(), 1000u);
    sim_destroy(sim);
}

TEST(BrunelNetwork, StdpChangesWeights) {
    Brunel b(200, 50, 5.0, true);
    auto before = b.conns[0]->connectivity.weights.clone();
    auto* sim = sim_create(b.region, SimulationOptions().dt_fast(1e-4).dt_slow(1e-4).dt_structural(1e-2));
    sim_run_steps(sim, 500);
    auto after = b.conns[0]->connectivity.weights;
    EXPECT_GT((after.to(torch::kCPU) - before.to(torch::kCPU)).abs().sum().item<float>(), 0.0f);
    EXPECT_LE(after.max().item<float>(), 5 * 500e-12 * 1.0001);
    sim_destroy(sim);
}

TEST(BrunelNetwork, InhibitionLowersRate) {
    double rates[2];
    int k = 0;
    for (double g : {1.0, 5.0}) {
        Brunel b(200, 50, g, false);
        auto* sim = sim_create(b.region, SimulationOptions().dt_fast(1e-4).duration(0.1));
        sim_record(sim, b.exc, {"spike"});
        sim_run(sim);
        rates[k++] = sim_get_spikes(sim, b.exc).size(0) / (200 * 0.1);
        sim_destroy(sim);
    }
    EXPECT_LE(rates[1], rates[0] + 20.0);
}

TEST(Simulation, RecordersCallbacksAndNoNaN) {
    auto* lif = neuron::lif_create(32, neuron::LIFOptions().i_bg(500e-12));
    auto pop = std::shared_ptr<Population>(population_create("p", neuron::lif_as_module(lif), 32, torch::kCUDA),
                                           population_destroy);
    auto* region = region_create("r");
    region_add_population(region, pop);
    auto* sim = sim_create(region, SimulationOptions().dt_fast(1e-4));
    sim_record(sim, pop, {"v", "spike"}, 2);
    int calls = 0;
    sim_add_callback(sim, 25, [&](const Simulation& s, double) {
        ++calls;
        EXPECT_EQ(s.clock.step() % 25, 0u);
    });
    sim_run_steps(sim, 200);
    EXPECT_EQ(calls, 7);   // steps 25, 50, ..., 175
    auto v = sim_get_recorded(sim, pop, "v");
    EXPECT_EQ(v.size(0), 100);
    EXPECT_EQ(v.size(1), 32);
    EXPECT_GT(sim_get_spikes(sim, pop).size(0), 0);
    EXPECT_FALSE(torch::any(torch::isnan(state_get(pop->state, "v"))).item<bool>());
    EXPECT_THROW(sim_get_spikes(sim, nullptr), c10::Error);
    sim_destroy(sim);
    region_destroy(region);
    neuron::lif_destroy(lif);
}

// State recorders read through device probes: the rows equal the state
// after each step, read directly, with sim_step calls and no host wait in
// between; spikes recorded by a sim_step loop equal those of sim_run_steps.
TEST(Simulation, ProbesEqualDirectReadsAndStepLoopEqualsRun) {
    auto make = [](neuron::LIFNeuron** out) {
        auto* lif = neuron::lif_create(64, neuron::LIFOptions().i_bg(500e-12));
        neuron::lif_to_device(lif, torch::kCUDA);
        lif->v.copy_(-0.065 + 0.01 * torch::arange(64, torch::TensorOptions().device(torch::kCUDA)) / 64.0);
        *out = lif;
        return std::shared_ptr<Population>(population_create("p", neuron::lif_as_module(lif), 64, torch::kCUDA),
                                           population_destroy);
    };
    neuron::LIFNeuron* l1 = nullptr;
    auto pop = make(&l1);
    auto* region = region_create("r");
    region_add_population(region, pop);
    auto* sim = sim_create(region, SimulationOptions().dt_fast(1e-4));
    sim_record(sim, pop, {"v", "spike"});
    // 300 steps: past the first spikes (about 140 steps from rest at this
    // drive) and past one probe ring of 256 rows
    std::vector<torch::Tensor> direct;
    for (int k = 0; k < 300; ++k) {
        sim_step(sim);
        direct.push_back(state_get(pop->state, "v").cpu().clone());
    }
    auto rec = sim_get_recorded(sim, pop, "v");
    ASSERT_TRUE(rec.size(0) == 300);
    for (int k = 0; k < 300; ++k) EXPECT_TRUE(torch::equal(rec[k], direct[k]));
    auto sp_steps = sim_get_spikes(sim, pop).clone();
    neuron::LIFNeuron* l2 = nullptr;
    auto pop2 = make(&l2);
    auto* region2 = region_create("r2");
    region_add_population(region2, pop2);
    auto* sim2 = sim_create(region2, SimulationOptions().dt_fast(1e-4));
    sim_record(sim2, pop2, {"spike"});
    sim_run_steps(sim2, 300);
    auto sp_run = sim_get_spikes(sim2, pop2);
    EXPECT_GT(sp_run.size(0), 0);
    EXPECT_TRUE(torch::equal(sp_steps, sp_run));
    sim_destroy(sim2);
    region_destroy(region2);
    neuron::lif_destroy(l2);
    sim_destroy(sim);
    region_destroy(region);
    neuron::lif_destroy(l1);
}

// A Simulation from a YAML file (nrn::config::load): populations with
// synapse channels and STDP, run on the GPU, spikes recorded.
TEST(Config, LoadAndRunSimulation) {
    const std::string path = std::string("/tmp/nrn_cfg_sim_") + std::to_string(::getpid()) + ".yaml";
    FILE* f = std::fopen(path.c_str(), "w");
    std::fputs(R"(name: yaml_net
seed: 3
simulation:
  dt_fast: 0.1ms
  dt_slow: 0.1ms
  duration: 20ms
populations:
  - name: exc
    model: LIF
    count: 400
    params: {v_rest: -65mV, v_thresh: -50mV, v_reset: -65mV, tau_m: 20ms, i_bg: 400pA}
  - name: inh
    model: LIF
    count: 100
    params: {v_rest: -65mV, v_thresh: -50mV, v_reset: -65mV, tau_m: 10ms, i_bg: 400pA}
connections:
  - source: exc
    target: exc
    probability: 0.1
    weight: 200pA
    block_size: 64
    synapse: exponential
    synapse_params: {tau_decay: 2ms}
    plasticity: stdp
    plasticity_params: {learning_rate: 1e-9, w_max: 400pA}
  - source: exc
    target: inh
    probability: 0.1
    weight: 200pA
    block_size: 64
    synapse: AMPA
    synapse_params: {tau_rise: 0.5ms, tau_decay: 3ms, e_rev: 0mV}
  - {source: inh, target: exc, probability: 0.1, weight: -800pA, block_size: 64}
record:
  - population: exc
    variables: [spike]
)",
               f);
    std::fclose(f);
    Simulation* sim = config::load(path);
    ASSERT_TRUE(sim != nullptr);
    sim_run(sim);
    auto exc = region_find_population(sim->region, "exc");
    auto sp = sim_get_spikes(sim, exc);
    EXPECT_GT(sp.size(0), 10);
    sim_destroy(sim);
    std::remove(path.c_str());
}

NRN_TEST_MAIN()
