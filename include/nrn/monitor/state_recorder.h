// nrn/monitor/state_recorder.h -- state variable recorder
// (reference: include/nrn/monitor/state_recorder.h:18-80).
#pragma once

#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

#include <torch/torch.h>

#include <nrn/core/state.h>
#include <nrn/core/types.h>
#include <nrn/monitor/recorder.h>

namespace nrn {

struct StateRecorderState {
    std::string pop_name;
    std::vector<std::string> variables;
    int64_t subsample = 1;
    int64_t call_count = 0;
    std::unordered_map<std::string, std::vector<torch::Tensor>> history;
    std::vector<float> times;
};

StateRecorderState* state_recorder_create(std::string pop_name, std::vector<std::string> variables,
                                          int64_t subsample = 1);
void state_recorder_destroy(StateRecorderState* s);
void state_recorder_record(void* self, const State& state, double t);
void state_recorder_reset(void* self);
const char* state_recorder_population_name(void* self);
// [T, N]
torch::Tensor state_recorder_get(const StateRecorderState* s, const std::string& variable);
torch::Tensor state_recorder_get_times(const StateRecorderState* s);
const std::vector<std::string>& state_recorder_variables(const StateRecorderState* s);

extern recorder_ops state_recorder_ops;

inline Recorder state_recorder_as_recorder(StateRecorderState* s) {
    return Recorder{static_cast<void*>(s), &state_recorder_ops};
}

}  // namespace nrn
