// nrn/simulation/spike_buffer.h -- dense spike delay ring
// (reference: include/nrn/simulation/spike_buffer.h:18-57).
//
// Kept for the API.  Inside sim_run the engine does not use it: spikes are
// kept as compacted id lists per step on the GPU.
#pragma once

#include <cstdint>

#include <torch/torch.h>

namespace nrn {

class SpikeBuffer {
public:
    SpikeBuffer(int64_t n, int64_t max_delay_steps, torch::Device device);

    void push(const torch::Tensor& spikes);
    torch::Tensor read(int64_t delay_steps) const;
    torch::Tensor read_batch(const torch::Tensor& delay_steps) const;
    void reset();

    int64_t max_delay() const { return max_delay_steps_; }
    int64_t size() const { return n_; }

private:
    torch::Tensor buffer_;   // [max_delay_steps, N]
    int64_t n_;
    int64_t max_delay_steps_;
    int64_t write_pos_ = 0;
};

}  // namespace nrn
