// nrn/core/types.h -- simulation time and SI unit literals.
// Same names and values as the reference's include/nrn/core/types.h:8-50.
#pragma once

#include <cstdint>

namespace nrn {

using Time = double;       // seconds since the start of the simulation
using Duration = double;   // seconds

namespace literals {

#define NRN_UNIT_LITERAL(suffix, scale) \
    constexpr double operator""_##suffix(long double x) { return static_cast<double>(x) * (scale); }

NRN_UNIT_LITERAL(s, 1.0)
NRN_UNIT_LITERAL(ms, 1e-3)
NRN_UNIT_LITERAL(us, 1e-6)
NRN_UNIT_LITERAL(V, 1.0)
NRN_UNIT_LITERAL(mV, 1e-3)
NRN_UNIT_LITERAL(A, 1.0)
NRN_UNIT_LITERAL(nA, 1e-9)
NRN_UNIT_LITERAL(pA, 1e-12)
NRN_UNIT_LITERAL(F, 1.0)
NRN_UNIT_LITERAL(pF, 1e-12)
NRN_UNIT_LITERAL(S, 1.0)
NRN_UNIT_LITERAL(nS, 1e-9)
NRN_UNIT_LITERAL(m, 1.0)
NRN_UNIT_LITERAL(um, 1e-6)
NRN_UNIT_LITERAL(uM, 1e-6)
NRN_UNIT_LITERAL(nM, 1e-9)

#undef NRN_UNIT_LITERAL

}  // namespace literals
}  // namespace nrn
