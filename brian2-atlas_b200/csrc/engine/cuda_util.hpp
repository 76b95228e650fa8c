// Error-checking helpers for the CUDA runtime, driver and NVRTC APIs.
#pragma once

#include <cuda_runtime.h>
#include <nvrtc.h>

#include <string>

#include "../common/ir.hpp"

namespace b2gpu {

inline void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw b2ir::Error(std::string(what) + ": " + cudaGetErrorString(e));
}

inline void nvrtc_check(nvrtcResult e, const char* what) {
  if (e != NVRTC_SUCCESS) throw b2ir::Error(std::string(what) + ": " + nvrtcGetErrorString(e));
}

}  // namespace b2gpu

#define B2_CUDA(call) ::b2gpu::cuda_check((call), #call)
#define B2_NVRTC(call) ::b2gpu::nvrtc_check((call), #call)
