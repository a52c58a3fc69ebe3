// nrn/monitor/spike_recorder.h -- spike event recorder
// (reference: include/nrn/monitor/spike_recorder.h:21-73).
//
// record() compacts the spike vector on the GPU and copies only the ids.
// Inside sim_run the engine fills the recorder from its device raster.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include <torch/torch.h>

#include <nrn/core/state.h>
#include <nrn/core/types.h>
#include <nrn/monitor/recorder.h>

namespace nrn {

struct SpikeRecorderState {
    std::string pop_name;
    int64_t subsample = 1;
    int64_t call_count = 0;
    std::vector<float> neuron_ids;
    std::vector<float> times;
};

SpikeRecorderState* spike_recorder_create(std::string pop_name, int64_t subsample = 1);
void spike_recorder_destroy(SpikeRecorderState* s);
void spike_recorder_record(void* self, const State& state, double t);
void spike_recorder_reset(void* self);
const char* spike_recorder_population_name(void* self);
// [K, 2] float: (neuron id, time)
torch::Tensor spike_recorder_get_spikes(const SpikeRecorderState* s);
torch::Tensor spike_recorder_get_spike_times(const SpikeRecorderState* s, int64_t neuron_id);
int64_t spike_recorder_spike_count(const SpikeRecorderState* s);

extern recorder_ops spike_recorder_ops;

inline Recorder spike_recorder_as_recorder(SpikeRecorderState* s) {
    return Recorder{static_cast<void*>(s), &spike_recorder_ops};
}

}  // namespace nrn
