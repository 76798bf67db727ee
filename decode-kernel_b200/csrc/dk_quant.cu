// dk_quant.cu -- the int4 group-128 format on the GPU: quantize + pack,
// unpack to int, dequantize.  Bit-exact with python/decode_kernel/quantize.py
// (quantize_and_pack :26-51, unpack_to_int :54-63, dequantize :66-78) as torch
// evaluates it on the CPU:
//   scale32 = max(amax / 7, 1e-8)          (IEEE fp32 division)
//   q       = clamp(rint(w / scale32), -7, 7)   (round half to even)
//   word    = OR_n (q_n & 0xF) << 4n           (low nibble first)
//   scale16 = fp16(scale32)                    (round to nearest even)
// With DK_QUANT_TORCH_CUDA_SCALE the first line becomes amax * fp32(1/7),
// which is what the same torch expression computes on a CUDA tensor (its
// division by a host scalar is a multiplication by the scalar's reciprocal).
//
// Layout of the work: one warp per 128-weight group; lane l holds weights
// 4l..4l+3 (one float4 load), so a lane pair covers one packed word.
#include "dk_device.cuh"
#include "dk_host.h"

namespace dk {
namespace {

constexpr int kQuantWarps = 8;

__global__ void __launch_bounds__(kQuantWarps * 32) k_quantize_pack(const float* __restrict__ w,
                                                                    int M, int K,
                                                                    uint32_t* __restrict__ packed,
                                                                    __half* __restrict__ scales,
                                                                    int torch_cuda_scale) {
  const int lane = threadIdx.x & 31;
  const int groups = K / kGroup;
  const long long gid = (long long)blockIdx.x * kQuantWarps + (threadIdx.x >> 5);
  if (gid >= (long long)M * groups) return;
  const long long row = gid / groups;
  const int G = (int)(gid % groups);
  const float4 v = *reinterpret_cast<const float4*>(w + row * K + (long long)G * kGroup + 4 * lane);
  // amax with NaN propagation (torch.amax propagates NaN).
  float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  bool nan = isnan(v.x) || isnan(v.y) || isnan(v.z) || isnan(v.w);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    nan = __any_sync(0xffffffffu, nan);
  }
  float s;
  if (nan) {
    s = __int_as_float(0x7fc00000);
  } else {
    s = torch_cuda_scale ? __fmul_rn(m, 1.0f / 7.0f) : __fdiv_rn(m, 7.0f);
    s = fmaxf(s, 1e-8f);
  }
  const float vv[4] = {v.x, v.y, v.z, v.w};
  uint32_t nib = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float r = rintf(__fdiv_rn(vv[i], s));
    r = fminf(fmaxf(r, -7.f), 7.f);
    const int q = isnan(r) ? 0 : (int)r;
    nib |= ((uint32_t)q & 0xFu) << (4 * i);
  }
  // Lanes 2j and 2j+1 hold the low and high halves of word j.
  const uint32_t hi = __shfl_down_sync(0xffffffffu, nib, 1);
  if ((lane & 1) == 0) {
    packed[row * (K / kNibbles) + (long long)G * kWordsPerGroup + (lane >> 1)] = nib | (hi << 16);
  }
  if (lane == 0) scales[row * groups + G] = __float2half_rn(s);
}

__global__ void k_unpack_to_int(const uint32_t* __restrict__ packed, long long words,
                                int4* __restrict__ q) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < words;
       i += (long long)gridDim.x * blockDim.x) {
    const uint32_t wd = packed[i];
    int v[8];
#pragma unroll
    for (int n = 0; n < 8; ++n) v[n] = (int)(wd << (28 - 4 * n)) >> 28;
    q[2 * i] = make_int4(v[0], v[1], v[2], v[3]);
    q[2 * i + 1] = make_int4(v[4], v[5], v[6], v[7]);
  }
}

__global__ void k_dequantize(const uint32_t* __restrict__ packed, const __half* __restrict__ scales,
                             long long words, float4* __restrict__ w) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < words;
       i += (long long)gridDim.x * blockDim.x) {
    const uint32_t wd = packed[i];
    const float s = __half2float(scales[i / kWordsPerGroup]);  // groups are row-aligned
    float v[8];
#pragma unroll
    for (int n = 0; n < 8; ++n) v[n] = (float)((int)(wd << (28 - 4 * n)) >> 28) * s;
    w[2 * i] = make_float4(v[0], v[1], v[2], v[3]);
    w[2 * i + 1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

int grid_for(long long n, int threads) {
  long long b = (n + threads - 1) / threads;
  const long long cap = (long long)sm_count(-1) * 16;
  if (b > cap) b = cap;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace
}  // namespace dk

using namespace dk;

extern "C" dk_status dk_quantize_pack(const float* w, int M, int K, int32_t* packed,
                                      uint16_t* scales, unsigned flags, void* stream) {
  if (M < 0 || K < 0 || K % DK_GROUP_SIZE != 0 || (flags & ~DK_QUANT_TORCH_CUDA_SCALE))
    return DK_ERR_INVALID_ARG;
  if (M == 0 || K == 0) return DK_OK;
  if (!w || !packed || !scales || !aligned16(w) || (reinterpret_cast<uintptr_t>(packed) & 3u) ||
      (reinterpret_cast<uintptr_t>(scales) & 1u))
    return DK_ERR_INVALID_ARG;
  const long long ngroups = (long long)M * (K / kGroup);
  const long long blocks = (ngroups + kQuantWarps - 1) / kQuantWarps;
  if (blocks > 0x7fffffffLL) return DK_ERR_INVALID_ARG;
  k_quantize_pack<<<(unsigned)blocks, kQuantWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      w, M, K, reinterpret_cast<uint32_t*>(packed), reinterpret_cast<__half*>(scales),
      (flags & DK_QUANT_TORCH_CUDA_SCALE) ? 1 : 0);
  return check_launch("k_quantize_pack");
}

extern "C" dk_status dk_unpack_to_int(const int32_t* packed, int M, int K, int32_t* q,
                                      void* stream) {
  if (M < 0 || K < 0 || K % DK_GROUP_SIZE != 0) return DK_ERR_INVALID_ARG;
  if (M == 0 || K == 0) return DK_OK;
  if (!packed || !q || !aligned16(q) || (reinterpret_cast<uintptr_t>(packed) & 3u))
    return DK_ERR_INVALID_ARG;
  const long long words = (long long)M * (K / kNibbles);
  k_unpack_to_int<<<grid_for(words, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint32_t*>(packed), words, reinterpret_cast<int4*>(q));
  return check_launch("k_unpack_to_int");
}

extern "C" dk_status dk_dequantize(const int32_t* packed, const uint16_t* scales, int M, int K,
                                   float* w, void* stream) {
  if (M < 0 || K < 0 || K % DK_GROUP_SIZE != 0) return DK_ERR_INVALID_ARG;
  if (M == 0 || K == 0) return DK_OK;
  if (!packed || !scales || !w || !aligned16(w) || (reinterpret_cast<uintptr_t>(packed) & 3u) ||
      (reinterpret_cast<uintptr_t>(scales) & 1u))
    return DK_ERR_INVALID_ARG;
  const long long words = (long long)M * (K / kNibbles);
  k_dequantize<<<grid_for(words, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint32_t*>(packed), reinterpret_cast<const __half*>(scales), words,
      reinterpret_cast<float4*>(w));
  return check_launch("k_dequantize");
}
