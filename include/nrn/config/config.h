// nrn/config/config.h -- YAML configuration (reference: include/nrn/config/config.h).
// Not implemented in the reference either (src/config/config.cpp:8-18 throws);
// kept so that code naming it compiles; both calls throw std::runtime_error.
#pragma once

#include <string>

#include <nrn/network/region.h>
#include <nrn/simulation/runner.h>

namespace nrn {
namespace config {

Simulation* load(const std::string& path);
Region* load_region(const std::string& path);

}  // namespace config
}  // namespace nrn
