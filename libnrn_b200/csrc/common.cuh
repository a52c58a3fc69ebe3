// common.cuh -- error reporting shared by the device layer.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "nrn_cuda.h"

namespace nrn {

// Sets the calling thread's last error message and returns the status.
nrn_status_t fail(nrn_status_t s, const std::string& msg);
nrn_status_t cuda_fail(cudaError_t e, const char* what);

}  // namespace nrn

#define NRN_CHECK_ARG(cond, msg)                                   \
    do {                                                           \
        if (!(cond)) return ::nrn::fail(NRN_ERR_INVALID, (msg));   \
    } while (0)

#define NRN_CUDA_TRY(expr)                                         \
    do {                                                           \
        cudaError_t e_ = (expr);                                   \
        if (e_ != cudaSuccess) return ::nrn::cuda_fail(e_, #expr); \
    } while (0)

#define NRN_TRY(expr)                                              \
    do {                                                           \
        nrn_status_t s_ = (expr);                                  \
        if (s_ != NRN_OK) return s_;                               \
    } while (0)
