// The reference's core, clock and spike-buffer suites re-expressed
// (tests/core/test_types.cpp, test_state.cpp, test_module.cpp,
// tests/simulation/test_clock.cpp, tests/simulation/test_spike_buffer.cpp).
// Host-only: runs without a GPU.
#include <nrn/nrn.h>
#include <nrn/config/config.h>

#include <unistd.h>

#include <cstdio>

#include "nrn_test.h"

using namespace nrn;

TEST(Types, TimeLiterals) {
    EXPECT_DOUBLE_EQ(1.0_s, 1.0);
    EXPECT_DOUBLE_EQ(1.0_ms, 1e-3);
    EXPECT_DOUBLE_EQ(1.0_us, 1e-6);
    EXPECT_DOUBLE_EQ(0.1_ms, 0.1 * 1e-3);
}

TEST(Types, ElectricalLiterals) {
    EXPECT_DOUBLE_EQ(1.0_mV, 1e-3);
    EXPECT_DOUBLE_EQ(1.0_V, 1.0);
    EXPECT_DOUBLE_EQ(1.0_nA, 1e-9);
    EXPECT_DOUBLE_EQ(1.0_pA, 1e-12);
    EXPECT_DOUBLE_EQ(250.0_pF, 250.0 * 1e-12);
    EXPECT_DOUBLE_EQ(30.0_nS, 30.0 * 1e-9);
    EXPECT_DOUBLE_EQ(1.0_um, 1e-6);
    EXPECT_DOUBLE_EQ(1.0_uM, 1e-6);
    EXPECT_DOUBLE_EQ(1.0_nM, 1e-9);
}

TEST(State, SetGetContainsRemove) {
    State s;
    EXPECT_FALSE(state_contains(s, "v"));
    state_set(s, "v", torch::ones({3}));
    EXPECT_TRUE(state_contains(s, "v"));
    EXPECT_EQ(state_get(s, "v").size(0), 3);
    EXPECT_TRUE(state_remove(s, "v"));
    EXPECT_FALSE(state_remove(s, "v"));
}

TEST(State, MissingKeyThrows) {
    State s;
    EXPECT_THROW(state_get(s, "nope"), c10::Error);
    const State& cs = s;
    EXPECT_THROW(state_get(cs, "nope"), c10::Error);
}

TEST(State, CreateAndKeys) {
    auto s = state_create({"v", "u"}, 5);
    EXPECT_EQ(state_keys(s).size(), 2u);
    EXPECT_TRUE(torch::all(state_get(s, "u") == 0).item<bool>());
}

namespace {
struct Counter {
    int64_t n = 7;
    int forwards = 0;
    int resets = 0;
};
void c_forward(void* self, State& st, double, double) {
    static_cast<Counter*>(self)->forwards++;
    state_set(st, "x", torch::zeros({static_cast<Counter*>(self)->n}));
}
void c_reset(void* self) { static_cast<Counter*>(self)->resets++; }
const char* c_vars_names[] = {"x"};
const char** c_vars(void*, int* n) {
    *n = 1;
    return c_vars_names;
}
int64_t c_size(void* self) { return static_cast<Counter*>(self)->n; }
void c_to(void*, torch::Device) {}
nrn_ops counter_ops = {c_forward, c_reset, c_vars, c_size, c_to};
}  // namespace

TEST(Module, Dispatch) {
    Counter c;
    NrnModule m{&c, &counter_ops};
    State st;
    nrn_forward(&m, st, 0.0, 1e-4);
    nrn_forward(&m, st, 0.0, 1e-4);
    nrn_reset(&m);
    EXPECT_EQ(c.forwards, 2);
    EXPECT_EQ(c.resets, 1);
    EXPECT_EQ(nrn_size(&m), 7);
    int count = 0;
    const char** names = nrn_state_vars(&m, &count);
    EXPECT_EQ(count, 1);
    EXPECT_EQ(std::string(names[0]), "x");
    EXPECT_TRUE(state_contains(st, "x"));
}

TEST(Options, FluentDefaults) {
    auto o = neuron::LIFOptions();
    EXPECT_DOUBLE_EQ(o.v_rest(), -0.065);
    EXPECT_DOUBLE_EQ(o.tau_m(), 0.010);
    auto p = o.tau_m(0.02).v_thresh(-0.04);
    EXPECT_DOUBLE_EQ(p.tau_m(), 0.02);
    EXPECT_DOUBLE_EQ(p.v_thresh(), -0.04);
    EXPECT_DOUBLE_EQ(neuron::AdExOptions().b(), 80.5e-12);
    EXPECT_DOUBLE_EQ(neuron::IzhikevichOptions().d(), 8.0);
    EXPECT_DOUBLE_EQ(STDPOptions().a_minus(), -0.012);
    EXPECT_EQ(ConnectOptions().block_size(), 256);
}

TEST(Clock, StepsAndTime) {
    Clock c(0.1e-3, 10e-3, 1.0);
    EXPECT_EQ(c.step(), 0u);
    EXPECT_DOUBLE_EQ(c.time(), 0.0);
    for (int i = 0; i < 25; ++i) c.advance_fast();
    EXPECT_EQ(c.step(), 25u);
    EXPECT_DOUBLE_EQ(c.time(), 25 * 0.1e-3);
    c.reset();
    EXPECT_EQ(c.step(), 0u);
}

TEST(Clock, Boundaries) {
    Clock c(1e-3, 5e-3, 20e-3);
    EXPECT_TRUE(c.is_slow_boundary());   // step 0
    EXPECT_TRUE(c.is_structural_boundary());
    int slow = 0, structural = 0;
    for (int i = 0; i < 40; ++i) {
        c.advance_fast();
        slow += c.is_slow_boundary();
        structural += c.is_structural_boundary();
    }
    EXPECT_EQ(slow, 8);
    EXPECT_EQ(structural, 2);
}

TEST(Clock, Validation) {
    EXPECT_THROW(Clock(0.0, 1.0, 1.0), std::invalid_argument);
    EXPECT_THROW(Clock(1e-3, -1.0, 1.0), std::invalid_argument);
    EXPECT_THROW(Clock(1e-3, 1e-4, 1.0), std::invalid_argument);
    EXPECT_THROW(Clock(1e-3, 2.5e-3, 1.0), std::invalid_argument);
    EXPECT_NO_THROW(Clock(1e-4, 1e-2, 1.0));
}

TEST(SpikeBuffer, RingSemantics) {
    SpikeBuffer buf(3, 4, torch::kCPU);
    EXPECT_EQ(buf.size(), 3);
    EXPECT_EQ(buf.max_delay(), 4);
    EXPECT_TRUE(torch::all(buf.read(1) == 0).item<bool>());   // read before push
    for (int k = 0; k < 3; ++k) {
        auto s = torch::zeros({3});
        s[k] = 1.0;
        buf.push(s);
    }
    EXPECT_FLOAT_EQ(buf.read(1)[2].item<float>(), 1.0f);
    EXPECT_FLOAT_EQ(buf.read(2)[1].item<float>(), 1.0f);
    EXPECT_FLOAT_EQ(buf.read(3)[0].item<float>(), 1.0f);
    EXPECT_TRUE(torch::all(buf.read(4) == 0).item<bool>());
    for (int k = 0; k < 4; ++k) buf.push(torch::full({3}, static_cast<float>(k + 10)));   // wrap around
    EXPECT_FLOAT_EQ(buf.read(1)[0].item<float>(), 13.0f);
    EXPECT_FLOAT_EQ(buf.read(4)[0].item<float>(), 10.0f);
    auto b = buf.read_batch(torch::tensor({1, 2, 4}, torch::kLong));
    EXPECT_FLOAT_EQ(b[0].item<float>(), 13.0f);
    EXPECT_FLOAT_EQ(b[1].item<float>(), 12.0f);
    EXPECT_FLOAT_EQ(b[2].item<float>(), 10.0f);
    EXPECT_THROW(buf.read(0), c10::Error);
    EXPECT_THROW(buf.read(5), c10::Error);
    EXPECT_THROW(buf.push(torch::zeros({4})), c10::Error);
    buf.reset();
    EXPECT_TRUE(torch::all(buf.read(1) == 0).item<bool>());
}

TEST(ConnectivityTensor, EffectiveWeightsCapacityDensity) {
    ConnectivityTensor ct;
    ct.block_index.row_ptr = torch::tensor({0, 1, 2}, torch::kInt32);
    ct.block_index.col_idx = torch::tensor({0, 1}, torch::kInt32);
    ct.block_size = 2;
    ct.n_source = 4;
    ct.n_target = 4;
    ct.weights = torch::full({2, 2, 2}, 2.0);
    ct.structural_mask = torch::tensor({1.f, 0.f, 1.f, 1.f, 0.f, 0.f, 1.f, 0.f}).reshape({2, 2, 2});
    ct.modulatory_mask = torch::full({2, 2, 2}, 0.5);
    auto e = ct.effective_weights();
    EXPECT_FLOAT_EQ(e[0][0][0].item<float>(), 1.0f);
    EXPECT_FLOAT_EQ(e[0][0][1].item<float>(), 0.0f);
    EXPECT_EQ(ct.total_capacity(), 8);
    EXPECT_EQ(ct.active_count(), 4);
    EXPECT_DOUBLE_EQ(ct.density(), 0.5);
    EXPECT_EQ(ct.block_index.find_block(1, 1), 1);
    EXPECT_EQ(ct.block_index.find_block(0, 1), -1);
    EXPECT_THROW(ct.block_index.find_block(2, 0), c10::Error);
}

TEST(Topology, RandomCsrInvariants) {
    torch::manual_seed(3);
    auto* topo = random_topology_create(RandomTopologyOptions().probability(0.2));
    auto gen = random_topology_as_generator(topo);
    auto ct = topology_generate(&gen, 100, 70, 16, torch::kCPU);
    auto rp = ct.block_index.row_ptr;
    EXPECT_EQ(rp.size(0), 5 + 1);
    EXPECT_EQ(rp[-1].item<int>(), ct.block_index.n_blocks());
    EXPECT_TRUE(torch::all(rp.slice(0, 1) >= rp.slice(0, 0, -1)).item<bool>());
    EXPECT_EQ(ct.weights.size(1), 16);
    EXPECT_TRUE(torch::all(ct.delays == 1).item<bool>());
    random_topology_destroy(topo);
}

// YAML configuration (nrn::config; a stub that throws in the reference,
// src/config/config.cpp:8-18): a Region from a file, and the errors.
static std::string write_tmp(const char* name, const char* text) {
    std::string path = std::string("/tmp/nrn_cfg_") + std::to_string(::getpid()) + "_" + name;
    FILE* f = std::fopen(path.c_str(), "w");
    std::fputs(text, f);
    std::fclose(f);
    return path;
}

TEST(Config, MissingFileThrows) {
    EXPECT_THROW(config::load("/nonexistent/x.yaml"), std::runtime_error);
    EXPECT_THROW(config::load_region("/nonexistent/x.yaml"), std::runtime_error);
}

TEST(Config, LoadRegion) {
    const std::string path = write_tmp("region.yaml", R"(# a small balanced network
name: cortex
seed: 7
simulation:
  dt_fast: 0.1ms
  device: cpu
populations:
- name: exc
  model: LIF
  count: 80
  params: {v_rest: 0mV, v_thresh: 20mV, v_reset: 10mV, tau_m: 20ms, i_bg: 300pA}
- name: inh
  model: Izhikevich
  count: 20
  params:
    a: 0.1
    d: 2
connections:
  - source: exc
    target: inh
    topology: random
    probability: 0.2
    weight: 250pA
    block_size: 16
    synapse: exponential
    synapse_params: {tau_decay: 5ms}
  - source: exc
    target: exc
    probability: 0.1
    block_size: 16
    plasticity: stdp
    plasticity_params: {a_plus: 0.01, w_max: 500pA}
)");
    Region* r = config::load_region(path);
    ASSERT_TRUE(r != nullptr);
    EXPECT_EQ(r->name, std::string("cortex"));
    EXPECT_EQ(r->populations.size(), 2u);
    EXPECT_EQ(r->connections.size(), 2u);
    EXPECT_EQ(region_total_size(r), 100);
    auto exc = region_find_population(r, "exc");
    ASSERT_TRUE(exc != nullptr);
    EXPECT_EQ(exc->module.ops, &neuron::lif_ops);
    auto* lif = static_cast<neuron::LIFNeuron*>(exc->module.impl);
    EXPECT_NEAR(lif->options.v_thresh(), 0.020, 1e-12);
    EXPECT_NEAR(lif->options.i_bg(), 300e-12, 1e-20);
    auto inh = region_find_population(r, "inh");
    EXPECT_EQ(inh->module.ops, &neuron::izh_ops);
    EXPECT_NEAR(static_cast<neuron::IzhikevichNeuron*>(inh->module.impl)->options.a(), 0.1, 1e-12);
    auto& c0 = r->connections[0];
    EXPECT_EQ(c0->synapse.ops, &synapse::exp_synapse_ops);
    EXPECT_EQ(c0->connectivity.block_size, 16);
    EXPECT_EQ(c0->plasticity_rules.size(), 0u);
    EXPECT_EQ(r->connections[1]->plasticity_rules.size(), 1u);
    EXPECT_EQ(r->connections[1]->synapse.ops, &synapse::static_synapse_ops);
    // seeded: the same file gives the same connectivity
    Region* r2 = config::load_region(path);
    EXPECT_TRUE(torch::equal(r->connections[0]->connectivity.structural_mask,
                             r2->connections[0]->connectivity.structural_mask));
    region_destroy(r2);
    region_destroy(r);
    std::remove(path.c_str());
}

TEST(Config, ErrorsNameTheLine) {
    auto expect_error = [](const char* body, const char* needle) {
        // populations on the host (no GPU needed); the line numbers below
        // count this first line
        const std::string text = std::string("simulation: {device: cpu}\n") + body;
        const std::string path = write_tmp("bad.yaml", text.c_str());
        bool ok = false;
        try {
            Region* r = config::load_region(path);
            region_destroy(r);
        } catch (const std::runtime_error& e) {
            ok = std::string(e.what()).find(needle) != std::string::npos;
            if (!ok) std::printf("    message: %s\n", e.what());
        }
        std::remove(path.c_str());
        EXPECT_TRUE(ok);
    };
    expect_error("populations:\n  - name: a\n    model: HH\n    count: 3\n", ":4: unknown neuron model 'HH'");
    expect_error("populations:\n  - name: a\n    model: LIF\n    count: 3\n    params: {tau_q: 1ms}\n",
                 "unknown field 'tau_q'");
    expect_error("populations:\n  - name: a\n    model: LIF\n    count: 3\nconnections:\n  - source: a\n"
                 "    target: b\n",
                 "no population 'b'");
    expect_error("populations:\n  - name: a\n    model: LIF\n    count: 3 apples\n", "unknown unit");
    expect_error("populations: [1, 2\n", "expected ','");
    expect_error("a: 1\na: 2\n", "duplicate key 'a'");
}

NRN_TEST_MAIN()
