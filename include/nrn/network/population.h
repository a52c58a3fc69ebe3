// nrn/network/population.h -- a named group of neurons sharing one model
// (reference: include/nrn/network/population.h:18-76).
#pragma once

#include <optional>
#include <string>

#include <torch/torch.h>

#include <nrn/core/module.h>
#include <nrn/core/state.h>
#include <nrn/core/types.h>

namespace nrn {

struct Population {
    std::string name;
    NrnModule module;   // the neuron model (not owned)
    State state;        // filled by the first forward; aliases the model's tensors
    int64_t n;
    std::optional<torch::Tensor> positions;
};

inline Population* population_create(const std::string& name, NrnModule module, int64_t n,
                                     torch::Device /*device*/) {
    TORCH_CHECK(n > 0, "Population '", name, "' must have at least 1 neuron");
    auto* pop = new Population();
    pop->name = name;
    pop->module = module;
    pop->n = n;
    return pop;
}

inline void population_destroy(Population* pop) { delete pop; }

inline void population_set_positions(Population* pop, torch::Tensor positions) {
    TORCH_CHECK(positions.dim() == 2 && positions.size(0) == pop->n && positions.size(1) == 3,
                "positions must have shape [", pop->n, ", 3], got ", positions.sizes());
    pop->positions = std::move(positions);
}

inline void population_to_device(Population* pop, torch::Device device) {
    state_to_device(pop->state, device);
    if (pop->positions.has_value()) pop->positions = pop->positions->to(device);
    nrn_to_device(&pop->module, device);
}

inline std::string population_repr(const Population* pop) {
    std::string r = "Population(name='" + pop->name + "', n=" + std::to_string(pop->n) + ", module=...)";
    if (pop->positions.has_value()) r += " with positions";
    return r;
}

}  // namespace nrn
