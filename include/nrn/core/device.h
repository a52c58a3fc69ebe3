// nrn/core/device.h -- device placement helpers (reference: include/nrn/core/device.h:11-31).
#pragma once

#include <torch/torch.h>

namespace nrn {

struct Device {
    static torch::Device GPU(int index = 0) { return torch::Device(torch::kCUDA, static_cast<c10::DeviceIndex>(index)); }
    static torch::Device CPU() { return torch::Device(torch::kCPU); }
    static torch::Device Default() { return torch::cuda::is_available() ? GPU(0) : CPU(); }
    static int64_t gpu_count() { return static_cast<int64_t>(torch::cuda::device_count()); }
};

}  // namespace nrn
