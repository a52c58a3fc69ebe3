// nrn/core/state.h -- named tensor bag (reference: include/nrn/core/state.h:12-75).
//
// Entries alias the model's own storage: the tensors a neuron publishes are
// its device state arrays, so writes through the map are seen by the engine.
#pragma once

#include <string>
#include <unordered_map>
#include <vector>

#include <torch/torch.h>

namespace nrn {

using State = std::unordered_map<std::string, torch::Tensor>;

inline void state_set(State& s, const std::string& name, torch::Tensor t) { s[name] = std::move(t); }

inline torch::Tensor& state_get(State& s, const std::string& name) {
    auto it = s.find(name);
    TORCH_CHECK(it != s.end(), "State does not contain tensor '", name, "'");
    return it->second;
}

inline const torch::Tensor& state_get(const State& s, const std::string& name) {
    auto it = s.find(name);
    TORCH_CHECK(it != s.end(), "State does not contain tensor '", name, "'");
    return it->second;
}

inline bool state_contains(const State& s, const std::string& name) { return s.find(name) != s.end(); }

inline bool state_remove(State& s, const std::string& name) { return s.erase(name) > 0; }

inline std::vector<std::string> state_keys(const State& s) {
    std::vector<std::string> keys;
    keys.reserve(s.size());
    for (const auto& kv : s) keys.push_back(kv.first);
    return keys;
}

inline void state_to_device(State& s, torch::Device device) {
    for (auto& kv : s) kv.second = kv.second.to(device);
}

inline State state_create(const std::vector<std::string>& var_names, int64_t n,
                          torch::Device device = torch::kCPU, torch::Dtype dtype = torch::kFloat32) {
    State s;
    const auto opts = torch::TensorOptions().device(device).dtype(dtype);
    for (const auto& name : var_names) s[name] = torch::zeros({n}, opts);
    return s;
}

}  // namespace nrn
