// Test infrastructure, not product code.
//
// A C ABI over the reference's own host entry points (RohanDisa/decode-kernel
// include/decode_kernel/gemv_w4a16.h:34-49, csrc/gemv_w4a16.cu:568-628), so
// that the GPU parity tests and the reference arm of bench.py can run the
// reference's unmodified CUDA kernels through ctypes on the same device
// buffers as this library.  oracle/Makefile's `ref` target compiles this file
// together with the reference's csrc/gemv_w4a16.cu, straight from the
// reference checkout and with the reference's own nvcc flags (setup.py:47-56)
// for sm_100a, into oracle/_ref/libdkref.so.  Nothing here is shipped.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "decode_kernel/gemv_w4a16.h"

extern "C" {

// decode_kernel::w4a16_gemv with the launch config spelled out as ints
// (the fields of GemvLaunchConfig, gemv_w4a16.h:27-32).  The workspace is the
// fp32 [B, M] buffer v4 accumulates into; the reference's binding passes it
// zero-filled (bindings.cpp:63-68), and so must the caller.  Returns the CUDA
// error state after the launch (the reference prints launch errors and clears
// them, so a failed launch shows here only through its output).
int dkref_gemv(const void* packed, const void* scales, const void* x, void* y, int M, int K,
               int B, int version, int split_k, int reuse_weights, int warps_per_row,
               void* workspace, void* stream) {
  decode_kernel::GemvLaunchConfig cfg;
  cfg.version = static_cast<decode_kernel::KernelVersion>(version);
  cfg.split_k = split_k;
  cfg.reuse_weights = reuse_weights != 0;
  cfg.warps_per_row = warps_per_row;
  decode_kernel::w4a16_gemv(static_cast<const uint32_t*>(packed),
                            static_cast<const __half*>(scales), static_cast<const __half*>(x),
                            static_cast<__half*>(y), M, K, B, cfg,
                            static_cast<float*>(workspace), static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaPeekAtLastError());
}

// The reference's dispatch stamp (gemv_w4a16.cu:558-564; synchronizes).
int dkref_last_kernel_stamp(void) { return decode_kernel::last_kernel_stamp(); }

}  // extern "C"
