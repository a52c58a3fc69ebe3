// nrn/monitor/recorder.h -- recorder handle (reference: include/nrn/monitor/recorder.h:15-52).
#pragma once

#include <string>

#include <nrn/core/state.h>
#include <nrn/core/types.h>

namespace nrn {

struct recorder_ops {
    void (*record)(void* self, const State& state, double t);
    void (*reset)(void* self);
    const char* (*population_name)(void* self);
};

struct Recorder {
    void* impl;
    recorder_ops* ops;
};

inline void recorder_record(Recorder* r, const State& state, double t) { r->ops->record(r->impl, state, t); }
inline void recorder_reset(Recorder* r) { r->ops->reset(r->impl); }
inline const char* recorder_population_name(Recorder* r) { return r->ops->population_name(r->impl); }

}  // namespace nrn
