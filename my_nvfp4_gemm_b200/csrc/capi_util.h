// capi_util.h — host-side helpers shared by the C-ABI entry points.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/nvfp4_b200.h"

namespace nvfp4 {

inline int status_from_cuda(cudaError_t e) { return e == cudaSuccess ? NVFP4_OK : NVFP4_ERR_CUDA; }

inline bool aligned_to(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// Streaming-multiprocessor count of the current device (cached per device).
int current_device_sm_count(int* device_out);

}  // namespace nvfp4
