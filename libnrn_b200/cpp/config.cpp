// config.cpp -- YAML configuration entry points; not implemented, as in the
// reference (src/config/config.cpp:8-18), which also throws.
#include <nrn/config/config.h>

#include <stdexcept>

namespace nrn {
namespace config {

Simulation* load(const std::string& path) {
    throw std::runtime_error("nrn::config::load: YAML configuration is not implemented (" + path + ")");
}

Region* load_region(const std::string& path) {
    throw std::runtime_error("nrn::config::load_region: YAML configuration is not implemented (" + path + ")");
}

}  // namespace config
}  // namespace nrn
