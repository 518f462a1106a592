// Launch-status bookkeeping shared by the host launchers.
#pragma once

#include <cuda_runtime.h>

#include "../../include/t4a_b200.h"

namespace t4a {
namespace runtime {

// Last CUDA error a launcher of this thread observed (reported by t4a_last_cuda_error).
int& last_error();

// Status of the launches just issued on this thread: T4A_ERR_CUDA when the runtime
// reports a launch error.
inline int check_launch() {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    last_error() = static_cast<int>(err);
    return T4A_ERR_CUDA;
  }
  return T4A_OK;
}

}  // namespace runtime
}  // namespace t4a
