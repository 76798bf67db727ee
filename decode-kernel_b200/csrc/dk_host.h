// dk_host.h -- host-side helpers shared by the library's translation units.
#pragma once

#include <algorithm>
#include <cstdint>

#include <cuda_runtime.h>

#include "dk_w4a16.h"

namespace dk {

// Records the CUDA error behind a DK_ERR_LAUNCH / DK_ERR_CUDA return so that
// dk_last_cuda_error() can report it (per host thread).
void set_cuda_error(cudaError_t e, const char* where);

// Number of SMs of `device` (-1 = current), cached per device.
int sm_count(int device);

// Current device id.
int current_device();

// Device address of the device error word on the current device (defined in
// dk_gemv.cu), for kernels of other translation units; nullptr on failure.
int* device_error_address();

inline dk_status check_launch(const char* where) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e, where);
    return DK_ERR_LAUNCH;
  }
  return DK_OK;
}

inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

}  // namespace dk
