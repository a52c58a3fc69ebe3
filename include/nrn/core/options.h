// nrn/core/options.h -- fluent option fields (reference: include/nrn/core/options.h:17-20).
//
//   struct Foo { NRN_ARG(double, tau, 0.02); };
//   Foo().tau(0.01).tau()  == 0.01
#pragma once

#include <torch/torch.h>

#define NRN_ARG(type, name, default_val)                                       \
    type name##_ = default_val;                                                \
    auto name() const -> type { return name##_; }                              \
    auto name(type val) -> decltype(*this)& {                                  \
        name##_ = val;                                                         \
        return *this;                                                          \
    }
