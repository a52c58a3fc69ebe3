// monitor.cpp -- spike and state recorders of the nrn:: API
// (src/monitor/spike_recorder.cpp, src/monitor/state_recorder.cpp).
//
// record() on a CUDA spike vector compacts it on the GPU and copies only
// the ids (the reference copies the whole vector and scans it on the host).
// Inside sim_run the engine fills spike recorders from its device raster.
#include <nrn/monitor/spike_recorder.h>
#include <nrn/monitor/state_recorder.h>

#include <algorithm>
#include <vector>

#include "support.h"

namespace nrn {

// --------------------------------------------------------- spikes ----

recorder_ops spike_recorder_ops = {spike_recorder_record, spike_recorder_reset, spike_recorder_population_name};

SpikeRecorderState* spike_recorder_create(std::string pop_name, int64_t subsample) {
    TORCH_CHECK(subsample >= 1, "spike_recorder_create: subsample must be >= 1, got ", subsample);
    auto* s = new SpikeRecorderState{};
    s->pop_name = std::move(pop_name);
    s->subsample = subsample;
    return s;
}

void spike_recorder_destroy(SpikeRecorderState* s) { delete s; }

namespace detail {

// Ascending indices of the non-zero entries of a spike vector.
std::vector<int32_t> spike_ids(const torch::Tensor& spikes) {
    std::vector<int32_t> ids;
    const int64_t n = spikes.numel();
    if (n == 0) return ids;
    if (spikes.is_cuda()) {
        auto x = spikes.to(torch::kFloat32).contiguous();
        auto dev = torch::TensorOptions().dtype(torch::kInt32).device(x.device());
        auto out = torch::empty({n}, dev);
        auto cnt = torch::zeros({1}, dev);
        check(nrn_cuda_compact(x.data_ptr<float>(), n, out.data_ptr<int32_t>(), cnt.data_ptr<int32_t>(),
                               stream_of(x)),
              "spike compaction");
        const int32_t k = cnt.item<int32_t>();
        auto host = out.slice(0, 0, k).to(torch::kCPU);
        ids.assign(host.data_ptr<int32_t>(), host.data_ptr<int32_t>() + k);
        std::sort(ids.begin(), ids.end());
    } else {
        auto x = spikes.to(torch::kFloat32).contiguous();
        const float* p = x.data_ptr<float>();
        for (int64_t i = 0; i < n; ++i)
            if (p[i] != 0.0f) ids.push_back(static_cast<int32_t>(i));
    }
    return ids;
}

}  // namespace detail

void spike_recorder_record(void* self, const State& state, double t) {
    auto* s = static_cast<SpikeRecorderState*>(self);
    ++s->call_count;
    if (s->call_count % s->subsample != 0) return;
    if (!state_contains(state, "spike")) return;
    for (int32_t id : detail::spike_ids(state_get(state, "spike"))) {
        s->neuron_ids.push_back(static_cast<float>(id));
        s->times.push_back(static_cast<float>(t));
    }
}

void spike_recorder_reset(void* self) {
    auto* s = static_cast<SpikeRecorderState*>(self);
    s->neuron_ids.clear();
    s->times.clear();
    s->call_count = 0;
}

const char* spike_recorder_population_name(void* self) { return static_cast<SpikeRecorderState*>(self)->pop_name.c_str(); }

torch::Tensor spike_recorder_get_spikes(const SpikeRecorderState* s) {
    const int64_t k = static_cast<int64_t>(s->neuron_ids.size());
    if (k == 0) return torch::zeros({0, 2}, torch::kFloat32);
    auto out = torch::empty({k, 2}, torch::kFloat32);
    float* p = out.data_ptr<float>();
    for (int64_t i = 0; i < k; ++i) {
        p[2 * i] = s->neuron_ids[i];
        p[2 * i + 1] = s->times[i];
    }
    return out;
}

torch::Tensor spike_recorder_get_spike_times(const SpikeRecorderState* s, int64_t neuron_id) {
    std::vector<float> m;
    const float target = static_cast<float>(neuron_id);
    for (size_t i = 0; i < s->neuron_ids.size(); ++i)
        if (s->neuron_ids[i] == target) m.push_back(s->times[i]);
    if (m.empty()) return torch::zeros({0}, torch::kFloat32);
    return torch::from_blob(m.data(), {static_cast<int64_t>(m.size())}, torch::kFloat32).clone();
}

int64_t spike_recorder_spike_count(const SpikeRecorderState* s) { return static_cast<int64_t>(s->neuron_ids.size()); }

// ---------------------------------------------------------- state ----

recorder_ops state_recorder_ops = {state_recorder_record, state_recorder_reset, state_recorder_population_name};

StateRecorderState* state_recorder_create(std::string pop_name, std::vector<std::string> variables,
                                          int64_t subsample) {
    TORCH_CHECK(subsample >= 1, "state_recorder_create: subsample must be >= 1, got ", subsample);
    auto* s = new StateRecorderState{};
    s->pop_name = std::move(pop_name);
    s->variables = std::move(variables);
    s->subsample = subsample;
    return s;
}

void state_recorder_destroy(StateRecorderState* s) { delete s; }

void state_recorder_record(void* self, const State& state, double t) {
    auto* s = static_cast<StateRecorderState*>(self);
    ++s->call_count;
    if (s->call_count % s->subsample != 0) return;
    for (const auto& var : s->variables)
        if (state_contains(state, var)) s->history[var].push_back(state_get(state, var).detach().cpu().clone());
    s->times.push_back(static_cast<float>(t));
}

void state_recorder_reset(void* self) {
    auto* s = static_cast<StateRecorderState*>(self);
    for (auto& kv : s->history) kv.second.clear();
    s->times.clear();
    s->call_count = 0;
}

const char* state_recorder_population_name(void* self) { return static_cast<StateRecorderState*>(self)->pop_name.c_str(); }

torch::Tensor state_recorder_get(const StateRecorderState* s, const std::string& variable) {
    auto it = s->history.find(variable);
    TORCH_CHECK(it != s->history.end(), "state_recorder_get: variable '", variable,
                "' is not being recorded for population '", s->pop_name, "'");
    if (it->second.empty()) return torch::zeros({0, 0}, torch::kFloat32);
    return torch::stack(it->second, 0);
}

torch::Tensor state_recorder_get_times(const StateRecorderState* s) {
    if (s->times.empty()) return torch::zeros({0}, torch::kFloat32);
    return torch::from_blob(const_cast<float*>(s->times.data()), {static_cast<int64_t>(s->times.size())},
                            torch::kFloat32)
        .clone();
}

const std::vector<std::string>& state_recorder_variables(const StateRecorderState* s) { return s->variables; }

}  // namespace nrn
