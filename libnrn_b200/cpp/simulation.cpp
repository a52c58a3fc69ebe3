// simulation.cpp -- Clock, SpikeBuffer and the simulation loop of the nrn:: API.
//
// sim_step's phases (src/simulation/runner.cpp:95-173) run in the device
// engine (include/nrn_cuda.h, nrn_engine_*): delivery of the spikes emitted
// d steps ago, the fused neuron updates, pair STDP at slow-clock boundaries
// and the spike raster.  The engine is built at the first step from the
// Region:
//   * populations: the neuron models' own tensors are the engine's state
//     (v, w/u, refractory, spike, I_syn), so State entries stay aliased;
//     parameters that are uniform are passed as scalars, others as arrays,
//     and re-examined whenever a parameter tensor changes (version counter);
//   * connections: the structurally present synapses of each
//     ConnectivityTensor (mask != 0, inside the valid block area) become a
//     per-synapse CSR with weight W, gain Ms*Mm and the delays tensor;
//   * plasticity: STDP rules attached to a connection run in the engine.
// Steps run in CUDA graphs between host events: callbacks, state
// recorders (which need a snapshot every step), and raster draining.  After
// a run the plastic weights are written back into the ConnectivityTensor.
#include <nrn/connectivity/connect.h>
#include <nrn/monitor/spike_recorder.h>
#include <nrn/monitor/state_recorder.h>
#include <nrn/neuron/adex.h>
#include <nrn/neuron/izhikevich.h>
#include <nrn/neuron/lif.h>
#include <nrn/plasticity/plasticity_rule.h>
#include <nrn/plasticity/stdp.h>
#include <nrn/simulation/runner.h>
#include <nrn/synapse/synapse.h>

#include <algorithm>
#include <map>
#include <cmath>
#include <stdexcept>
#include <vector>

#include "support.h"

namespace nrn {

// --------------------------------------------------------------- Clock ----

Clock::Clock(Duration dt_fast, Duration dt_slow, Duration dt_structural)
    : dt_fast_(dt_fast), dt_slow_(dt_slow), dt_structural_(dt_structural), current_time_(0.0), fast_step_(0) {
    if (dt_fast_ <= 0.0) throw std::invalid_argument("dt_fast must be positive");
    if (dt_slow_ <= 0.0) throw std::invalid_argument("dt_slow must be positive");
    if (dt_structural_ <= 0.0) throw std::invalid_argument("dt_structural must be positive");
    const double rs = dt_slow_ / dt_fast_, rt = dt_structural_ / dt_fast_;
    slow_ratio_ = static_cast<uint64_t>(std::round(rs));
    structural_ratio_ = static_cast<uint64_t>(std::round(rt));
    if (slow_ratio_ == 0) throw std::invalid_argument("dt_slow must be >= dt_fast");
    if (structural_ratio_ == 0) throw std::invalid_argument("dt_structural must be >= dt_fast");
    constexpr double tol = 1e-6;
    if (std::abs(rs - static_cast<double>(slow_ratio_)) > tol)
        throw std::invalid_argument("dt_slow must be an integer multiple of dt_fast");
    if (std::abs(rt - static_cast<double>(structural_ratio_)) > tol)
        throw std::invalid_argument("dt_structural must be an integer multiple of dt_fast");
}

void Clock::advance_fast() {
    ++fast_step_;
    current_time_ = static_cast<double>(fast_step_) * dt_fast_;
}

bool Clock::is_slow_boundary() const { return fast_step_ % slow_ratio_ == 0; }
bool Clock::is_structural_boundary() const { return fast_step_ % structural_ratio_ == 0; }

void Clock::reset() {
    fast_step_ = 0;
    current_time_ = 0.0;
}

// --------------------------------------------------------- SpikeBuffer ----

SpikeBuffer::SpikeBuffer(int64_t n, int64_t max_delay_steps, torch::Device device)
    : n_(n), max_delay_steps_(max_delay_steps), write_pos_(0) {
    TORCH_CHECK(n > 0, "SpikeBuffer: n must be positive");
    TORCH_CHECK(max_delay_steps > 0, "SpikeBuffer: max_delay_steps must be positive");
    buffer_ = torch::zeros({max_delay_steps, n}, torch::TensorOptions().dtype(torch::kFloat32).device(device));
}

void SpikeBuffer::push(const torch::Tensor& spikes) {
    TORCH_CHECK(spikes.dim() == 1 && spikes.size(0) == n_, "SpikeBuffer::push: expected 1-D tensor of size ", n_,
                ", got shape ", spikes.sizes());
    buffer_[write_pos_ % max_delay_steps_].copy_(spikes);
    ++write_pos_;
}

torch::Tensor SpikeBuffer::read(int64_t delay_steps) const {
    TORCH_CHECK(delay_steps >= 1 && delay_steps <= max_delay_steps_, "SpikeBuffer::read: delay_steps must be in [1, ",
                max_delay_steps_, "], got ", delay_steps);
    if (write_pos_ < delay_steps) return torch::zeros({n_}, buffer_.options());
    return buffer_[(write_pos_ - delay_steps) % max_delay_steps_];
}

torch::Tensor SpikeBuffer::read_batch(const torch::Tensor& delay_steps) const {
    TORCH_CHECK(delay_steps.dim() == 1 && delay_steps.size(0) == n_,
                "SpikeBuffer::read_batch: expected 1-D int64 tensor of size ", n_, ", got shape ",
                delay_steps.sizes());
    auto d = delay_steps.to(buffer_.device(), torch::kLong).contiguous();
    if (buffer_.is_cuda()) {
        auto out = torch::empty({n_}, buffer_.options());
        detail::check(nrn_cuda_gather_ring(buffer_.data_ptr<float>(), n_, max_delay_steps_, write_pos_,
                                           d.data_ptr<int64_t>(), out.data_ptr<float>(), detail::stream_of(out)),
                      "SpikeBuffer::read_batch");
        return out;
    }
    auto row = (torch::full({n_}, write_pos_, d.options()) - d).remainder(max_delay_steps_);
    return buffer_.index({row, torch::arange(n_, d.options())});
}

void SpikeBuffer::reset() {
    buffer_.zero_();
    write_pos_ = 0;
}

// ------------------------------------------------------------ engine ----

struct SimEngine {
    nrn_engine* e = nullptr;
    int device = 0;
    struct Pop {
        std::shared_ptr<Population> pop;
        int model = 0;
        int32_t id = 0;
        int64_t offset = 0;
        std::vector<torch::Tensor> params;
        std::vector<uint32_t> versions;
        std::vector<const void*> data;
        std::vector<void*> state;   // v, aux, refractory, spike, I_syn pointers given to the engine
    };
    struct Conn {
        Connection* conn = nullptr;
        int32_t proj = -1;
        int64_t nnz = 0;
        bool plastic = false;
        float w_min = 0.0f, w_max = 0.0f;
        torch::Tensor coo_pos;   // flat index into [n_blocks, B, B] of each synapse
        torch::Tensor valid;     // in-range entries (the reference clamps these)
        torch::Tensor w_dev;     // plastic: [n_blocks, B, B] float32 on the engine's device
        torch::Tensor w_buf;     // plastic: [nnz] the engine's weights in synapse order
        bool aliased = false;    // ConnectivityTensor::weights is w_dev itself
    };
    // A state recorder's variable, copied on the device at every step into
    // a ring of probe_depth rows (nrn_engine_add_probe).
    struct Probe {
        StateRecorderState* rec = nullptr;
        std::string var;
        int32_t pop = 0;
        torch::Tensor ring;      // [probe_depth, n]
    };
    std::vector<Pop> pops;
    std::vector<Conn> conns;
    std::vector<Probe> probes;
    int32_t probe_depth = 0;
    size_t n_pops = 0, n_conns = 0;
    std::vector<int32_t> raster_step, raster_gid;
    // steps run and not yet read back (spike raster, probes), and whether
    // the plastic weights changed since the last write-back
    int64_t pending_first = 0, pending_steps = 0;
    bool weights_dirty = false;
    // the engine's window, and the most steps between raster reads that
    // cannot overflow the raster (every recorded neuron spiking every step)
    int64_t window = 1, raster_every = 64;
    // orders the engine stream after the caller's stream and back
    cudaEvent_t order_ev = nullptr;

    ~SimEngine() {
        if (order_ev) cudaEventDestroy(order_ev);
        if (e) nrn_engine_destroy(e);
    }
};

namespace {

int model_of(const NrnModule& m) {
    if (m.ops == &neuron::lif_ops) return NRN_MODEL_LIF;
    if (m.ops == &neuron::adex_ops) return NRN_MODEL_ADEX;
    if (m.ops == &neuron::izh_ops) return NRN_MODEL_IZH;
    TORCH_CHECK(false, "sim: population model is not one of LIF, AdEx, Izhikevich");
    return -1;
}

// The tensors of a model that the engine reads, in the engine's slot order.
void model_tensors(SimEngine::Pop& p, std::vector<torch::Tensor*>& st, std::vector<torch::Tensor*>& par) {
    NrnModule& m = p.pop->module;
    if (p.model == NRN_MODEL_LIF) {
        auto* x = static_cast<neuron::LIFNeuron*>(m.impl);
        st = {&x->v, nullptr, &x->refractory, &x->spike, &x->I_syn};
        par = {&x->v_rest, &x->v_thresh, &x->v_reset, &x->tau_m, &x->tau_ref, &x->c_m, &x->i_bg};
    } else if (p.model == NRN_MODEL_ADEX) {
        auto* x = static_cast<neuron::AdExNeuron*>(m.impl);
        st = {&x->v, &x->w, &x->refractory, &x->spike, &x->I_syn};
        par = {&x->v_rest, &x->v_thresh, &x->v_reset, &x->v_peak, &x->tau_m, &x->tau_w, &x->tau_ref,
               &x->c_m, &x->g_l, &x->a, &x->b, &x->delta_t, &x->i_bg};
    } else {
        auto* x = static_cast<neuron::IzhikevichNeuron*>(m.impl);
        st = {&x->v, &x->u, nullptr, &x->spike, &x->I_syn};
        par = {&x->a, &x->b, &x->c, &x->d, &x->v_peak};
    }
}

// Uniform parameters become scalars, others stay per-neuron arrays.
void param_slots(SimEngine::Pop& p, const std::vector<torch::Tensor*>& par, const float** arr, float* uni) {
    p.params.clear();
    p.versions.clear();
    p.data.clear();
    for (size_t k = 0; k < par.size(); ++k) {
        torch::Tensor& t = *par[k];
        float* ptr = detail::cuda_f32(t, p.pop->n, "parameter", "sim");
        auto mm = torch::aminmax(t);
        const float lo = std::get<0>(mm).item<float>(), hi = std::get<1>(mm).item<float>();
        if (lo == hi) {
            arr[k] = nullptr;
            uni[k] = lo;
        } else {
            arr[k] = ptr;
            uni[k] = 0.0f;
        }
        p.params.push_back(t);
        p.versions.push_back(t._version());
        p.data.push_back(t.data_ptr());
    }
}

bool wants_spikes(const Simulation* sim, const std::string& name) {
    for (const auto& r : sim->recorders)
        if (r.ops == &spike_recorder_ops && name == r.ops->population_name(r.impl)) return true;
    return false;
}

void build_engine(Simulation* sim) {
    Region* region = sim->region;
    TORCH_CHECK(region != nullptr, "sim: no region");
    auto eng = std::make_shared<SimEngine>();
    // device of the first population's state
    TORCH_CHECK(!region->populations.empty(), "sim: the region has no populations");
    {
        SimEngine::Pop probe;
        probe.pop = region->populations.front();
        probe.model = model_of(probe.pop->module);
        std::vector<torch::Tensor*> st, par;
        model_tensors(probe, st, par);
        TORCH_CHECK(st[0]->is_cuda(), "sim: population state must be on a CUDA device (libnrn_b200 has no CPU path)");
        eng->device = st[0]->device().index();
    }
    detail::check(nrn_engine_create(&eng->e, eng->device, sim->options.dt_fast(),
                                    static_cast<int32_t>(sim->clock.slow_ratio())),
                  "sim: engine");
    int64_t offset = 0;
    for (auto& pp : region->populations) {
        SimEngine::Pop p;
        p.pop = pp;
        p.model = model_of(pp->module);
        p.offset = offset;
        std::vector<torch::Tensor*> st, par;
        model_tensors(p, st, par);
        nrn_pop_desc_t d{};
        d.model = p.model;
        d.n = static_cast<int32_t>(pp->n);
        d.gid_offset = static_cast<int32_t>(offset);
        d.record = wants_spikes(sim, pp->name) ? 1 : 0;
        float* ptr[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
        for (int k = 0; k < 5; ++k)
            if (st[k]) ptr[k] = detail::cuda_f32(*st[k], pp->n, "state", "sim");
        d.v = ptr[0];
        d.aux = ptr[1];
        d.refractory = ptr[2];
        d.spike = ptr[3];
        d.i_syn = ptr[4];
        p.state.assign(ptr, ptr + 5);
        param_slots(p, par, d.param, d.uniform);
        detail::check(nrn_engine_add_population(eng->e, &d, &p.id), "sim: add population");
        offset += pp->n;
        eng->pops.push_back(std::move(p));
    }
    auto pop_index = [&](const std::shared_ptr<Population>& pp) {
        for (size_t i = 0; i < eng->pops.size(); ++i)
            if (eng->pops[i].pop == pp) return static_cast<int32_t>(i);
        TORCH_CHECK(false, "sim: connection endpoint '", pp->name, "' is not a population of the region");
        return -1;
    };
    const torch::Device dev(torch::kCUDA, static_cast<c10::DeviceIndex>(eng->device));
    // Synapse modules of the connections (Connection::synapse) become synapse
    // channels of their target population: one channel per distinct
    // (model, time constants, reversal) on a population; static synapses
    // (or none) deliver into I_syn directly.
    std::vector<std::vector<nrn_syn_desc_t>> chans(eng->pops.size());
    auto receptor_of = [&](const NrnModule& m, int32_t tgt) -> int32_t {
        nrn_syn_desc_t d{};
        if (m.ops == &synapse::exp_synapse_ops && m.impl) {
            const auto& o = static_cast<synapse::ExponentialSynapse*>(m.impl)->options;
            d.kind = NRN_SYN_EXP;
            d.tau_decay = o.tau_decay();
        } else if (m.ops == &synapse::dexp_synapse_ops && m.impl) {
            const auto& o = static_cast<synapse::DoubleExponentialSynapse*>(m.impl)->options;
            d.kind = NRN_SYN_DEXP;
            d.tau_rise = o.tau_rise();
            d.tau_decay = o.tau_decay();
        } else if (m.ops == &synapse::ampa_ops && m.impl) {
            const auto& o = static_cast<synapse::AMPASynapse*>(m.impl)->options;
            d.kind = NRN_SYN_AMPA;
            d.tau_rise = o.tau_rise();
            d.tau_decay = o.tau_decay();
            d.e_rev = o.e_rev();
        } else {
            return NRN_RECV_CURRENT;
        }
        auto& list = chans[static_cast<size_t>(tgt)];
        for (size_t k = 0; k < list.size(); ++k)
            if (list[k].kind == d.kind && list[k].tau_rise == d.tau_rise && list[k].tau_decay == d.tau_decay &&
                list[k].e_rev == d.e_rev)
                return NRN_RECV_CHANNEL + static_cast<int32_t>(k);
        int32_t ch = 0;
        detail::check(nrn_engine_add_synapse_channel(eng->e, eng->pops[static_cast<size_t>(tgt)].id, &d, &ch),
                      "sim: synapse channel");
        list.push_back(d);
        return NRN_RECV_CHANNEL + ch;
    };
    for (auto& cp : region->connections) {
        Connection* c = cp.get();
        auto& ct = c->connectivity;
        SimEngine::Conn cc;
        cc.conn = c;
        const int64_t B = ct.block_size;
        const int64_t nb = ct.block_index.n_blocks();
        auto i64 = torch::TensorOptions().dtype(torch::kLong).device(dev);
        // (block, row, col) of every present synapse inside the valid area
        auto mask = ct.structural_mask.to(dev).to(torch::kFloat32).reshape({nb, B, B});
        auto rp = ct.block_index.row_ptr.to(dev).to(torch::kLong);
        auto ci = ct.block_index.col_idx.to(dev).to(torch::kLong);
        auto blk = torch::arange(nb, i64);
        auto row_of_blk = torch::searchsorted(rp, blk, false, true) - 1;   // right=true
        auto t_base = (row_of_blk * B).view({nb, 1, 1});
        auto s_base = (ci.slice(0, 0, nb) * B).view({nb, 1, 1});
        auto ar = torch::arange(B, i64);
        auto tgt_all = t_base + ar.view({1, B, 1});
        auto src_all = s_base + ar.view({1, 1, B});
        cc.valid = (tgt_all < ct.n_target) & (src_all < ct.n_source);
        auto present = (mask != 0) & cc.valid;
        auto flat = present.reshape({-1}).nonzero().reshape({-1});
        cc.coo_pos = flat;
        cc.nnz = flat.numel();
        auto src = src_all.expand({nb, B, B}).reshape({-1}).index_select(0, flat).to(torch::kInt32);
        auto tgt = tgt_all.expand({nb, B, B}).reshape({-1}).index_select(0, flat).to(torch::kInt32);
        auto W = ct.weights.to(dev).to(torch::kFloat32).reshape({-1}).index_select(0, flat).contiguous();
        auto gain = (mask * ct.modulatory_mask.to(dev).to(torch::kFloat32).reshape({nb, B, B}))
                        .reshape({-1})
                        .index_select(0, flat)
                        .contiguous();
        const bool unit_gain = cc.nnz == 0 || (gain == 1.0f).all().item<bool>();
        torch::Tensor delay;
        if (ct.delays.defined()) {
            auto d = ct.delays.to(dev).to(torch::kLong).reshape({-1}).index_select(0, flat);
            if (cc.nnz > 0) {
                const int64_t dmin = d.min().item<int64_t>(), dmax = d.max().item<int64_t>();
                TORCH_CHECK(dmin >= 1, "sim: synaptic delays must be >= 1 step");
                TORCH_CHECK(dmax <= sim->options.max_delay_steps() && dmax <= 255, "sim: delay of ", dmax,
                            " steps exceeds max_delay_steps (", sim->options.max_delay_steps(), ")");
            }
            delay = d.to(torch::kUInt8).contiguous();
        } else {
            delay = torch::ones({cc.nnz}, torch::TensorOptions().dtype(torch::kUInt8).device(dev));
        }
        src = src.contiguous();
        tgt = tgt.contiguous();
        nrn_proj_desc_t pd{};
        pd.src_pop = pop_index(c->source);
        pd.tgt_pop = pop_index(c->target);
        pd.receptor = receptor_of(c->synapse, pd.tgt_pop);
        pd.on_device = 1;
        pd.nnz = cc.nnz;
        pd.src = src.data_ptr<int32_t>();
        pd.tgt = tgt.data_ptr<int32_t>();
        pd.w = W.data_ptr<float>();
        pd.delay = delay.data_ptr<uint8_t>();
        pd.mod = unit_gain ? nullptr : gain.data_ptr<float>();
        torch::cuda::synchronize(eng->device);
        detail::check(nrn_engine_add_projection(eng->e, &pd, &cc.proj), "sim: add connection");
        for (auto& rule : c->plasticity_rules) {
            TORCH_CHECK(rule.ops == &stdp_ops, "sim: only STDP plasticity rules run in the engine");
            const STDPOptions& o = static_cast<STDPState*>(rule.impl)->opts;
            const double p[7] = {o.tau_plus(), o.tau_minus(), o.a_plus(), o.a_minus(), o.w_min(), o.w_max(),
                                 o.learning_rate()};
            detail::check(nrn_engine_set_stdp(eng->e, cc.proj, p), "sim: STDP");
            cc.plastic = true;
            cc.w_min = static_cast<float>(o.w_min());
            cc.w_max = static_cast<float>(o.w_max());
            TORCH_CHECK(c->plasticity_rules.size() == 1, "sim: one plasticity rule per connection");
        }
        eng->conns.push_back(std::move(cc));
    }
    // Plastic weights stay on the device between steps: w_dev is the block
    // tensor the engine's weights are written back into (clamped once now,
    // as the reference clamps every in-range entry at each update); it
    // becomes ConnectivityTensor::weights when that already lives on this
    // device as float32.
    for (auto& cc : eng->conns) {
        if (!cc.plastic) continue;
        auto& ct = cc.conn->connectivity;
        auto W = ct.weights.to(dev).to(torch::kFloat32).contiguous().clone();
        cc.w_dev = torch::where(cc.valid, W.clamp(cc.w_min, cc.w_max), W).contiguous();
        cc.w_buf = torch::empty({std::max<int64_t>(cc.nnz, 1)}, torch::TensorOptions().dtype(torch::kFloat32).device(dev));
        cc.aliased = ct.weights.is_cuda() && ct.weights.device() == dev && ct.weights.scalar_type() == torch::kFloat32;
        if (cc.aliased) ct.weights = cc.w_dev.view(ct.weights.sizes());
    }
    // state recorders: device probes, read back every probe_depth steps
    for (auto& r : sim->recorders) {
        if (r.ops != &state_recorder_ops) continue;
        auto* sr = static_cast<StateRecorderState*>(r.impl);
        for (size_t i = 0; i < eng->pops.size(); ++i) {
            auto& p = eng->pops[i];
            if (p.pop->name != sr->pop_name) continue;
            for (const auto& var : sr->variables) {
                int slot = -1;
                if (var == "v") slot = NRN_VAR_V;
                else if ((var == "w" && p.model == NRN_MODEL_ADEX) || (var == "u" && p.model == NRN_MODEL_IZH))
                    slot = NRN_VAR_AUX;
                else if (var == "refractory" && p.model != NRN_MODEL_IZH) slot = NRN_VAR_REFRACTORY;
                else if (var == "spike") slot = NRN_VAR_SPIKE;
                else if (var == "I_syn") slot = NRN_VAR_ISYN;
                if (slot < 0) continue;   // not in the model's state: not recorded (state_contains)
                if (eng->probe_depth == 0) {
                    int64_t tot = 0;
                    for (auto& q : eng->pops) tot += q.pop->n;
                    eng->probe_depth = static_cast<int32_t>(std::max<int64_t>(8, std::min<int64_t>(256, (int64_t(1) << 26) / std::max<int64_t>(tot, 1))));
                }
                SimEngine::Probe pr;
                pr.rec = sr;
                pr.var = var;
                pr.pop = static_cast<int32_t>(i);
                pr.ring = torch::empty({eng->probe_depth, p.pop->n}, torch::TensorOptions().dtype(torch::kFloat32).device(dev));
                detail::check(nrn_engine_add_probe(eng->e, p.id, slot, pr.ring.data_ptr<float>(), eng->probe_depth, nullptr),
                              "sim: state probe");
                eng->probes.push_back(std::move(pr));
            }
        }
    }
    // sim_create already ran the initialising update (forward with dt = 0)
    detail::check(nrn_engine_finalize(eng->e, 0), "sim: finalize");
    // continue the clock's step numbering (slow-clock boundaries, raster)
    detail::check(nrn_engine_set_step(eng->e, static_cast<int64_t>(sim->clock.step())), "sim: step");
    nrn_engine_info_t info{};
    detail::check(nrn_engine_info(eng->e, &info), "sim: engine info");
    eng->window = std::max<int64_t>(1, info.window);
    if (info.recorded_neurons > 0) eng->raster_every = std::max<int64_t>(1, info.raster_capacity / info.recorded_neurons);
    TORCH_CHECK(cudaEventCreateWithFlags(&eng->order_ev, cudaEventDisableTiming) == cudaSuccess, "sim: cudaEventCreate");
    eng->n_pops = region->populations.size();
    eng->n_conns = region->connections.size();
    sim->engine = eng;
}

// Re-reads parameter tensors and state pointers that the user changed.
void refresh(Simulation* sim) {
    SimEngine& g = *sim->engine;
    for (auto& p : g.pops) {
        std::vector<torch::Tensor*> st, par;
        model_tensors(p, st, par);
        bool changed = false;
        for (size_t k = 0; k < par.size(); ++k)
            changed = changed || par[k]->_version() != p.versions[k] || par[k]->data_ptr() != p.data[k];
        if (changed) {
            const float* arr[NRN_MAX_PARAMS] = {nullptr};
            float uni[NRN_MAX_PARAMS] = {0.0f};
            param_slots(p, par, arr, uni);
            detail::check(nrn_engine_set_params(g.e, p.id, arr, uni), "sim: parameters");
        }
        float* ptr[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
        for (int k = 0; k < 5; ++k)
            if (st[k]) ptr[k] = detail::cuda_f32(*st[k], p.pop->n, "state", "sim");
        if (!std::equal(ptr, ptr + 5, p.state.begin())) {
            detail::check(nrn_engine_set_state(g.e, p.id, ptr[0], ptr[1], ptr[2], ptr[3], ptr[4]), "sim: state");
            p.state.assign(ptr, ptr + 5);
        }
        // the engine does not read state["..."] entries; keep them aliased
        state_set(p.pop->state, "v", *st[0]);
        state_set(p.pop->state, "spike", *st[3]);
        state_set(p.pop->state, "I_syn", *st[4]);
        if (st[1]) state_set(p.pop->state, p.model == NRN_MODEL_ADEX ? "w" : "u", *st[1]);
        if (st[2]) state_set(p.pop->state, "refractory", *st[2]);
    }
}

void drain_raster(Simulation* sim, int64_t first_step, int64_t n_steps) {
    SimEngine& g = *sim->engine;
    bool any = false;
    for (auto& r : sim->recorders) any = any || r.ops == &spike_recorder_ops;
    if (!any) return;
    // one call into the host buffers; a second only when they must grow
    // (the call reports the count without copying)
    int64_t n = 0;
    const auto cap = static_cast<int64_t>(g.raster_step.size());
    nrn_status_t st = nrn_engine_raster(g.e, g.raster_step.data(), g.raster_gid.data(), cap, &n);
    if (st == NRN_ERR_CAPACITY && n > cap) {
        g.raster_step.resize(n + n / 2);
        g.raster_gid.resize(n + n / 2);
        st = nrn_engine_raster(g.e, g.raster_step.data(), g.raster_gid.data(),
                               static_cast<int64_t>(g.raster_step.size()), &n);
    }
    detail::check(st, "sim: raster");
    // each spike recorder counts its calls per step and keeps every
    // subsample-th step's spikes (spike_recorder.cpp semantics)
    const double dt = sim->options.dt_fast();
    for (auto& r : sim->recorders) {
        if (r.ops != &spike_recorder_ops) continue;
        auto* sr = static_cast<SpikeRecorderState*>(r.impl);
        const SimEngine::Pop* pop = nullptr;
        for (auto& p : g.pops)
            if (p.pop->name == sr->pop_name) pop = &p;
        if (!pop) {
            sr->call_count += n_steps;   // records nothing for an unknown population
            continue;
        }
        int64_t k = 0;
        for (int64_t step = first_step; step < first_step + n_steps; ++step) {
            ++sr->call_count;
            const bool keep = sr->call_count % sr->subsample == 0;
            while (k < n && g.raster_step[k] < step) ++k;
            for (; k < n && g.raster_step[k] == step; ++k) {
                const int64_t gid = g.raster_gid[k];
                if (!keep || gid < pop->offset || gid >= pop->offset + pop->pop->n) continue;
                sr->neuron_ids.push_back(static_cast<float>(gid - pop->offset));
                sr->times.push_back(static_cast<float>(static_cast<double>(step) * dt));
            }
        }
    }
}

// The plastic weights into the ConnectivityTensors: the engine's weights in
// synapse order (its own kernels, on the engine stream) scattered into w_dev
// -- no allocation, no host wait.  Only a connectivity kept off this device
// (or in another dtype) is then copied, which waits.
void sync_weights(Simulation* sim) {
    SimEngine& g = *sim->engine;
    if (!g.weights_dirty) return;
    nrn_stream_t es = nullptr;
    detail::check(nrn_engine_stream(g.e, &es), "sim");
    bool host_copy = false;
    for (auto& c : g.conns) {
        if (!c.plastic || c.nnz == 0) continue;
        detail::check(nrn_engine_weights_device(g.e, c.proj, c.w_buf.data_ptr<float>(), c.nnz), "sim: weights");
        detail::check(nrn_cuda_scatter(c.w_buf.data_ptr<float>(), c.coo_pos.data_ptr<int64_t>(), c.nnz,
                                       c.w_dev.data_ptr<float>(), es),
                      "sim: weight write-back");
        host_copy = host_copy || !c.aliased;
    }
    if (host_copy) {
        detail::check(nrn_engine_sync(g.e), "sim");
        for (auto& c : g.conns) {
            if (!c.plastic || c.aliased) continue;
            auto& ct = c.conn->connectivity;
            ct.weights.copy_(c.w_dev.view(ct.weights.sizes()));
        }
    }
    g.weights_dirty = false;
}

// Reads back what the steps run since the last call recorded: the spike
// raster into the spike recorders, the probe rows into the state recorders
// (one host wait).
void drain(Simulation* sim) {
    SimEngine& g = *sim->engine;
    if (g.pending_steps == 0) return;
    drain_raster(sim, g.pending_first, g.pending_steps);   // waits for the engine stream
    if (!g.probes.empty()) {
        detail::check(nrn_engine_sync(g.e), "sim");
        const double dt = sim->options.dt_fast();
        std::map<StateRecorderState*, std::vector<SimEngine::Probe*>> by_rec;
        for (auto& pr : g.probes) by_rec[pr.rec].push_back(&pr);
        for (auto& kv : by_rec) {
            StateRecorderState* sr = kv.first;
            std::vector<torch::Tensor> host;
            for (auto* pr : kv.second) host.push_back(pr->ring.cpu());
            for (int64_t s = g.pending_first; s < g.pending_first + g.pending_steps; ++s) {
                ++sr->call_count;
                if (sr->call_count % sr->subsample != 0) continue;
                const int64_t row = s % g.probe_depth;
                for (size_t k = 0; k < kv.second.size(); ++k)
                    sr->history[kv.second[k]->var].push_back(host[k][row].clone());
                sr->times.push_back(static_cast<float>(static_cast<double>(s) * dt));
            }
        }
    }
    g.pending_first += g.pending_steps;
    g.pending_steps = 0;
}

// Runs n steps.  No host wait per step: the spike raster and the state
// probes are read back when a callback or a query needs them, before the
// probe rings or the raster can fill (at window boundaries where the limit
// allows, so the engine replays whole-window graphs), and at the end of a
// multi-step call, which also writes the plastic weights back (bulk=true);
// sim_step leaves both on the device until then.
void run_steps(Simulation* sim, int64_t n, bool bulk) {
    if (n <= 0) return;
    Region* region = sim->region;
    if (!sim->engine || sim->engine->n_pops != region->populations.size() ||
        sim->engine->n_conns != region->connections.size()) {
        if (sim->engine) {
            drain(sim);
            sync_weights(sim);
        }
        sim->engine.reset();
        build_engine(sim);
        sim->engine->pending_first = static_cast<int64_t>(sim->clock.step());
    }
    SimEngine& g = *sim->engine;
    refresh(sim);
    nrn_stream_t es = nullptr;
    detail::check(nrn_engine_stream(g.e, &es), "sim");
    // the engine stream starts after the caller's queued work
    cudaEvent_t ev = g.order_ev;
    cudaEventRecord(ev, c10::cuda::getCurrentCUDAStream(g.device).stream());
    cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(es), ev, 0);
    const int64_t chunk = sim->options.use_cuda_graphs() ? 50 : 1;
    bool any_spike_rec = false;
    for (auto& r : sim->recorders) any_spike_rec = any_spike_rec || r.ops == &spike_recorder_ops;
    bool plastic = false;
    for (auto& c : g.conns) plastic = plastic || c.plastic;
    int64_t done = 0;
    while (done < n) {
        const int64_t step = static_cast<int64_t>(sim->clock.step());
        // a callback fires after step k (k > 0, k % every == 0): the segment
        // ends there so the callback sees that step's state
        int64_t seg = n - done;
        for (auto& cb : sim->callbacks) {
            const int64_t every = cb.first;
            const int64_t first = std::max<int64_t>(step, 1);
            const int64_t k = ((first + every - 1) / every) * every;
            seg = std::min(seg, k - step + 1);
        }
        // the next read-back: within the probe ring and the raster bound of
        // the first step not yet read, rounded down to a window boundary
        int64_t limit = 0;
        if (!g.probes.empty()) limit = g.probe_depth;
        if (any_spike_rec) limit = limit > 0 ? std::min(limit, g.raster_every) : g.raster_every;
        int64_t read_at = -1;
        if (limit > 0) {
            read_at = g.pending_first + limit;
            const int64_t aligned = read_at / g.window * g.window;
            if (aligned > step) read_at = aligned;
            seg = std::min(seg, read_at - step);
        }
        seg = std::max<int64_t>(seg, 1);
        detail::check(nrn_engine_run(g.e, seg, static_cast<int32_t>(std::min(seg, chunk))), "sim: run");
        g.pending_steps += seg;
        g.weights_dirty = g.weights_dirty || plastic;
        for (int64_t k = 0; k < seg; ++k) {
            const int64_t s_k = step + k;
            const double t = sim->clock.time();
            bool first_cb = true;
            for (auto& cb : sim->callbacks)
                if (s_k > 0 && s_k % cb.first == 0) {
                    if (first_cb) drain(sim);   // the callback sees the recorders up to this step
                    first_cb = false;
                    cb.second(*sim, t);
                }
            sim->clock.advance_fast();
        }
        if (read_at >= 0 && static_cast<int64_t>(sim->clock.step()) >= read_at) drain(sim);
        done += seg;
    }
    if (bulk) {
        drain(sim);
        sync_weights(sim);
    }
    // the caller's stream continues after the engine's work
    cudaEventRecord(ev, reinterpret_cast<cudaStream_t>(es));
    cudaStreamWaitEvent(c10::cuda::getCurrentCUDAStream(g.device).stream(), ev, 0);
}

}  // namespace

// -------------------------------------------------------- Simulation ----

Simulation* sim_create(Region* region, SimulationOptions options) {
    auto* sim = new Simulation();
    sim->region = region;
    sim->options = options;
    sim->clock = Clock(options.dt_fast(), options.dt_slow(), options.dt_structural());
    // The engine keeps spikes as compacted per-step id lists on the GPU, so
    // no dense SpikeBuffer is created per population.
    if (region)
        for (auto& pop : region->populations) nrn_forward(&pop->module, pop->state, 0.0, 0.0);
    return sim;
}

void sim_destroy(Simulation* sim) {
    if (sim && sim->engine) {
        drain(sim);
        sync_weights(sim);
    }
    delete sim;
}

void sim_sync(Simulation* sim) {
    TORCH_CHECK(sim != nullptr, "sim_sync: null simulation");
    if (!sim->engine) return;
    drain(sim);
    sync_weights(sim);
    detail::check(nrn_engine_sync(sim->engine->e), "sim_sync");
}

void sim_record(Simulation* sim, std::shared_ptr<Population> population, std::vector<std::string> variables,
                int64_t subsample) {
    TORCH_CHECK(population != nullptr, "Cannot record a null population");
    bool spikes = false;
    std::vector<std::string> vars;
    for (auto& v : variables) {
        if (v == "spike") spikes = true;
        else vars.push_back(std::move(v));
    }
    if (spikes) sim->recorders.push_back(spike_recorder_as_recorder(spike_recorder_create(population->name, subsample)));
    if (!vars.empty())
        sim->recorders.push_back(
            state_recorder_as_recorder(state_recorder_create(population->name, std::move(vars), subsample)));
    if (sim->engine) {
        // the raster flags and state probes are fixed at engine build:
        // rebuild to record this population
        drain(sim);
        sync_weights(sim);
        sim->engine.reset();
    }
}

void sim_run(Simulation* sim) {
    const auto n = static_cast<int64_t>(std::round(sim->options.duration() / sim->options.dt_fast()));
    sim_run_steps(sim, n);
}

void sim_run_steps(Simulation* sim, int64_t n) { run_steps(sim, n, true); }

void sim_step(Simulation* sim) { run_steps(sim, 1, false); }

torch::Tensor sim_get_spikes(const Simulation* sim, const std::shared_ptr<Population>& population) {
    TORCH_CHECK(population != nullptr, "Cannot query spikes for null population");
    if (sim->engine) drain(const_cast<Simulation*>(sim));
    for (const auto& r : sim->recorders)
        if (r.ops == &spike_recorder_ops && population->name == r.ops->population_name(r.impl))
            return spike_recorder_get_spikes(static_cast<SpikeRecorderState*>(r.impl));
    TORCH_CHECK(false, "No spike recorder registered for population '", population->name, "'");
    return {};
}

torch::Tensor sim_get_recorded(const Simulation* sim, const std::shared_ptr<Population>& population,
                               const std::string& variable) {
    TORCH_CHECK(population != nullptr, "Cannot query recorded data for null population");
    if (sim->engine) drain(const_cast<Simulation*>(sim));
    for (const auto& r : sim->recorders)
        if (r.ops == &state_recorder_ops && population->name == r.ops->population_name(r.impl))
            return state_recorder_get(static_cast<StateRecorderState*>(r.impl), variable);
    TORCH_CHECK(false, "No state recorder registered for population '", population->name, "' variable '", variable,
                "'");
    return {};
}

void sim_add_callback(Simulation* sim, int64_t every_n, SimCallback fn) {
    TORCH_CHECK(every_n > 0, "Callback interval must be positive");
    sim->callbacks.emplace_back(every_n, std::move(fn));
}

}  // namespace nrn
