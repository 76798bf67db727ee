// dk_stream.cu -- STREAM-style HBM probes for sm_100a: the read roof that is
// the GEMV metric's denominator, plus write and copy ceilings.
//
// Reference roles: d2d_copy_kernel, stream_read_kernel, stream_write_kernel and
// stream_recommended_blocks (csrc/gemv_w4a16.cu:421-425, 493-551, 593-626).
// The read probe keeps 8 independent 128-bit loads in flight per thread on the
// non-coherent, no-L1-allocate path, so each SM has ~256 KB outstanding --
// far more than HBM3e latency x bandwidth per SM needs.
#include "dk_device.cuh"
#include "dk_host.h"

namespace dk {
namespace {

constexpr int kStreamThreads = 256;
constexpr int kReadUnroll = 8;

__device__ __forceinline__ float sum4(const uint4& v) {
  return __uint_as_float(v.x) + __uint_as_float(v.y) + __uint_as_float(v.z) +
         __uint_as_float(v.w);
}

__global__ void __launch_bounds__(kStreamThreads) k_stream_read(const uint4* __restrict__ src,
                                                                float* __restrict__ partials,
                                                                size_t n) {
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  float acc[kReadUnroll];
#pragma unroll
  for (int u = 0; u < kReadUnroll; ++u) acc[u] = 0.f;
  size_t i = tid;
  for (; i + (kReadUnroll - 1) * stride < n; i += kReadUnroll * stride) {
    uint4 v[kReadUnroll];
#pragma unroll
    for (int u = 0; u < kReadUnroll; ++u) v[u] = ldg_stream(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < kReadUnroll; ++u) acc[u] += sum4(v[u]);
  }
  for (; i < n; i += stride) acc[0] += sum4(ldg_stream(src + i));
  float local = 0.f;
#pragma unroll
  for (int u = 0; u < kReadUnroll; ++u) local += acc[u];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
  __shared__ float red[kStreamThreads / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < kStreamThreads / 32; ++w) s += red[w];
    partials[blockIdx.x] = s;
  }
}

__global__ void __launch_bounds__(kStreamThreads) k_stream_write(float4* __restrict__ dst,
                                                                 size_t n) {
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const float4 one = make_float4(1.f, 1.f, 1.f, 1.f);
  for (size_t i = tid; i < n; i += stride) __stcs(dst + i, one);
}

__global__ void __launch_bounds__(kStreamThreads) k_d2d_copy(const uint4* __restrict__ src,
                                                             uint4* __restrict__ dst, size_t n) {
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = tid;
  for (; i + 3 * stride < n; i += 4 * stride) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = ldg_stream(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < 4; ++u) dst[i + u * stride] = v[u];
  }
  for (; i < n; i += stride) dst[i] = ldg_stream(src + i);
}

}  // namespace
}  // namespace dk

using namespace dk;

extern "C" int dk_stream_recommended_blocks(int device) {
  int blocks = sm_count(device) * 32;
  if (blocks < 1024) blocks = 1024;
  if (blocks > 8192) blocks = 8192;
  return blocks;
}

extern "C" dk_status dk_stream_read(const void* src, float* partials, size_t bytes, int blocks,
                                    void* stream) {
  if ((bytes & 15u) || !src || !partials || !aligned16(src)) return DK_ERR_INVALID_ARG;
  if (blocks < 1) blocks = dk_stream_recommended_blocks(-1);
  k_stream_read<<<blocks, kStreamThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), partials, bytes / 16);
  return check_launch("k_stream_read");
}

extern "C" dk_status dk_stream_write(void* dst, size_t bytes, int blocks, void* stream) {
  if ((bytes & 15u) || !dst || !aligned16(dst)) return DK_ERR_INVALID_ARG;
  if (blocks < 1) blocks = dk_stream_recommended_blocks(-1);
  k_stream_write<<<blocks, kStreamThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<float4*>(dst), bytes / 16);
  return check_launch("k_stream_write");
}

extern "C" dk_status dk_d2d_copy(const void* src, void* dst, size_t bytes, void* stream) {
  if ((bytes & 15u) || !src || !dst || !aligned16(src) || !aligned16(dst))
    return DK_ERR_INVALID_ARG;
  if (bytes == 0) return DK_OK;
  const size_t n = bytes / 16;
  const int blocks = dk_stream_recommended_blocks(-1);
  k_d2d_copy<<<blocks, kStreamThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), n);
  return check_launch("k_d2d_copy");
}
