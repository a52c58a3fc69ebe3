// nrn/simulation/clock.h -- multi-rate simulation clock
// (reference: include/nrn/simulation/clock.h:18-80, src/simulation/clock.cpp).
#pragma once

#include <cstdint>

#include <nrn/core/types.h>

namespace nrn {

class Clock {
public:
    Clock() : dt_fast_(0), dt_slow_(0), dt_structural_(0), slow_ratio_(1), structural_ratio_(1) {}
    // dt_slow and dt_structural must be integer multiples of dt_fast
    // (std::invalid_argument otherwise).
    Clock(Duration dt_fast, Duration dt_slow, Duration dt_structural);

    Time time() const { return current_time_; }
    uint64_t step() const { return fast_step_; }
    Duration dt_fast() const { return dt_fast_; }
    Duration dt_slow() const { return dt_slow_; }
    Duration dt_structural() const { return dt_structural_; }

    void advance_fast();
    bool is_slow_boundary() const;
    bool is_structural_boundary() const;
    void reset();

    uint64_t slow_ratio() const { return slow_ratio_; }

private:
    Duration dt_fast_;
    Duration dt_slow_;
    Duration dt_structural_;
    Time current_time_ = 0.0;
    uint64_t fast_step_ = 0;
    uint64_t slow_ratio_;
    uint64_t structural_ratio_;
};

}  // namespace nrn
