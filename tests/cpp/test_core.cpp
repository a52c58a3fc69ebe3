// The reference's core, clock and spike-buffer suites re-expressed
// (tests/core/test_types.cpp, test_state.cpp, test_module.cpp,
// tests/simulation/test_clock.cpp, tests/simulation/test_spike_buffer.cpp).
// Host-only: runs without a GPU.
#include <nrn/nrn.h>

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

TEST(Config, NotImplementedThrows) {
    EXPECT_THROW(config::load("x.yaml"), std::runtime_error);
    EXPECT_THROW(config::load_region("x.yaml"), std::runtime_error);
}

NRN_TEST_MAIN()
