// dk_abi.cu -- host utilities behind the C ABI: status text, per-thread CUDA
// error text, SM counts per device, version string.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "dk_host.h"

namespace dk {

namespace {
thread_local char g_err[256] = "no error";
std::mutex g_sm_mu;
int g_sm_cache[64] = {0};
}  // namespace

void set_cuda_error(cudaError_t e, const char* where) {
  std::snprintf(g_err, sizeof(g_err), "%s: %s (%s)", where, cudaGetErrorName(e),
                cudaGetErrorString(e));
}

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return 0;
  return d;
}

int sm_count(int device) {
  if (device < 0) device = current_device();
  if (device < 64) {
    std::lock_guard<std::mutex> lk(g_sm_mu);
    if (g_sm_cache[device] > 0) return g_sm_cache[device];
  }
  int sms = 1;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      sms < 1)
    sms = 1;
  if (device < 64) {
    std::lock_guard<std::mutex> lk(g_sm_mu);
    g_sm_cache[device] = sms;
  }
  return sms;
}

}  // namespace dk

extern "C" const char* dk_status_string(dk_status s) {
  switch (s) {
    case DK_OK:
      return "ok";
    case DK_ERR_INVALID_ARG:
      return "invalid argument (shape, range or alignment)";
    case DK_ERR_UNSUPPORTED:
      return "unsupported configuration";
    case DK_ERR_LAUNCH:
      return "kernel launch failed";
    case DK_ERR_TIMEOUT:
      return "bounded device wait timed out";
    case DK_ERR_CUDA:
      return "CUDA runtime call failed";
    case DK_ERR_WORKSPACE:
      return "workspace missing or too small";
  }
  return "unknown status";
}

extern "C" const char* dk_last_cuda_error(void) { return dk::g_err; }

extern "C" const char* dk_version(void) { return "decode-kernel-b200 0.1.0 sm_100a"; }
