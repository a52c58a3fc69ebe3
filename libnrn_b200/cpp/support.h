// support.h -- helpers shared by the nrn:: implementation files.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include <c10/cuda/CUDAStream.h>
#include <torch/torch.h>

#include "nrn_cuda.h"

namespace nrn {
namespace detail {

// Raises c10::Error (the reference's error type) for a failed device call.
inline void check(nrn_status_t st, const char* what) {
    TORCH_CHECK(st == NRN_OK, what, ": ", nrn_status_string(st), ": ", nrn_last_error());
}

inline nrn_stream_t stream_of(const torch::Tensor& t) {
    return reinterpret_cast<nrn_stream_t>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

// Float32, contiguous, on a CUDA device, n elements; rewrites `t` when it
// has to be made contiguous.  Returns the device pointer.
inline float* cuda_f32(torch::Tensor& t, int64_t n, const char* name, const char* where) {
    TORCH_CHECK(t.defined(), where, ": ", name, " is undefined");
    TORCH_CHECK(t.is_cuda(), where, ": ", name,
                " is on the CPU; libnrn_b200 runs the step on CUDA devices only (move the model with *_to_device)");
    TORCH_CHECK(t.scalar_type() == torch::kFloat32, where, ": ", name, " must be float32");
    TORCH_CHECK(t.numel() == n, where, ": ", name, " must have ", n, " elements, has ", t.numel());
    if (!t.is_contiguous()) t = t.contiguous();
    return t.data_ptr<float>();
}

inline torch::Device default_device() {
    if (torch::cuda::is_available()) {
        int dev = 0;
        cudaGetDevice(&dev);
        return torch::Device(torch::kCUDA, static_cast<c10::DeviceIndex>(dev));
    }
    return torch::Device(torch::kCPU);
}

}  // namespace detail
}  // namespace nrn
