// dk_gemv.cu -- the W4A16 GEMV kernel family for B200 (sm_100a) and its
// C-ABI entry point dk_w4a16_gemv.
//
// y[b, m] = sum_k x[b, k] * q[m, k] * scale[m, k / 128]
//
// The reference's family (csrc/gemv_w4a16.cu) is six plain-SIMT variants plus
// a multi-warp diagnostic, a split-K path and a batch weight-reuse path.  Each
// keeps its place in the API (same version numbers and stamps) but is a new
// kernel built around how B200 moves bytes:
//
//   v0  k_row_scalar    one thread per row (the reference's v0 role: the
//                       simplest correct kernel), LOP3 unpack, fp32 FMA.
//   v1  k_warp_row      one warp per row, 128-bit coalesced loads, fp32 FMA;
//       k_block_row     with warps_per_row > 1: one block per row.
//   v2  k_tile<Direct>  16-row tiles on the tensor pipe: LOP3 unpack straight
//                       into HMMA A fragments, fp32 accumulation, a 4-deep
//                       register prefetch of 128-bit weight loads.
//   v3  k_tile<Scales>  v2 with the tile's fp16 scales staged in shared memory.
//   v4  k_tile<SplitK>  v2 split along K over gridDim.y; partials go to a
//                       workspace and the last CTA of a tile sums them in
//                       split order (deterministic, one launch).
//   v5  k_stream        persistent CTAs, one per SM: a producer warp streams
//                       the CTA's contiguous row block into a 6-stage shared
//                       memory ring with 1-D bulk async copies (TMA engine,
//                       mbarrier transaction counts); 8 consumer warps unpack
//                       and feed HMMA.  The default and fastest path.
//   15  k_stream<reuse> the batch weight-reuse path: the same pipeline; every
//                       weight byte is read from HBM once and applied to up to
//                       32 batch rows per pass (mma N = 8 per tile).
//
// Why HMMA at batch 1: the dot product needs fp32 accumulation (the 1e-2
// tolerance does not survive fp16 accumulation at K = 11008), and doing it on
// CUDA cores costs ~2 extra instructions per weight.  One m16n8k16 does 256
// weights x up to 8 batch columns with fp32 accumulation in one issue slot, so
// the instruction budget per weight is ~1.3 (9 for the unpack of 8 weights),
// well under the ~2.6 B200 can issue per weight at HBM speed.
#include <algorithm>
#include <atomic>
#include <cstdio>

#define DK_DEVICE_GLOBALS
#include "dk_device.cuh"
#include "dk_host.h"

namespace dk {

struct GemvParams {
  const uint32_t* packed;  // [M, K/8]
  const __half* scales;    // [M, K/128]
  const __half* x;         // [B, K]
  __half* y;               // [B, M]
  int M, K, B;
  float* ws;               // v4: [K/128][B][M] fp32 per-group products
  unsigned* counters;      // v4: one arrival counter per 16-row tile
};

// ---------------------------------------------------------------------------
// Shared math
// ---------------------------------------------------------------------------

// fp32 dot of 8 unpacked weights (pairs (q0,q4),(q1,q5),(q2,q6),(q3,q7)) with
// x0..x7.
__device__ __forceinline__ float dot8_f32(const uint32_t (&h)[4], const uint4& xr, float acc) {
  uint32_t px[4];
  pair_x8(xr, px);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&px[i]));
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
  }
  return acc;
}

// x fragment loads for one group: thread (g, c) of a warp needs
// x[nt*8 + g][kx + 8t .. kx + 8t + 7], t = 0..3, kx = 128*G + 32*c.
template <int NT>
__device__ __forceinline__ void load_x_group(const __half* __restrict__ x, int K, int B, int kx,
                                             int g, uint4 (&xr)[NT][4]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int b = nt * 8 + g;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      xr[nt][t] = (b < B) ? ldg_keep(x + (size_t)b * K + kx + 8 * t) : make_uint4(0, 0, 0, 0);
    }
  }
}

// One group (128 k) of a 16-row tile: thread (g, c) holds words 4c..4c+3 of
// the group for rows g (wa) and g+8 (wb).  Eight HMMAs; the quad's four
// threads supply the 16 k of each one, all inside this group, so the group
// scale can be applied to the fp32 result afterwards.
template <int NT>
__device__ __forceinline__ void group_mma(const uint4& wa, const uint4& wb,
                                          const uint4 (&xr)[NT][4], float (&d)[NT][4]) {
  const uint32_t A[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t Bw[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    uint32_t ha[4], hb[4];
    unpack_q8(A[t], ha);
    unpack_q8(Bw[t], hb);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      uint32_t px[4];
      pair_x8(xr[nt][t], px);
      mma16816(d[nt], ha[0], hb[0], ha[1], hb[1], px[0], px[1]);
      mma16816(d[nt], ha[2], hb[2], ha[3], hb[3], px[2], px[3]);
    }
  }
}

// Canonical reduction order, shared by v2, v3, v4, v5 and the reuse path so
// that all of them return the same bits for the same inputs (and y[b] does
// not depend on which other batch rows or output rows are in the call):
//   a_G      = fp32(scale[m, G] * D_G)   (D_G: the group's HMMA dot product)
//   acc_w    = (((0 + a_w) + a_{w+8}) + a_{w+16}) + ...     for w = 0..7
//   y        = fp16_rn((((0 + acc_0) + acc_1) + ...) + acc_7)
// Explicit _rn intrinsics keep the compiler from contracting mul+add.
template <int NT>
__device__ __forceinline__ void scale_accumulate(float (&acc)[NT][4], const float (&d)[NT][4],
                                                 float sa, float sb) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    acc[nt][0] = __fadd_rn(acc[nt][0], __fmul_rn(sa, d[nt][0]));
    acc[nt][1] = __fadd_rn(acc[nt][1], __fmul_rn(sa, d[nt][1]));
    acc[nt][2] = __fadd_rn(acc[nt][2], __fmul_rn(sb, d[nt][2]));
    acc[nt][3] = __fadd_rn(acc[nt][3], __fmul_rn(sb, d[nt][3]));
  }
}

// D-fragment accumulators of one warp into red[16][8*NT].
template <int NT>
__device__ __forceinline__ void store_fragment(float* red, const float (&acc)[NT][4], int g,
                                               int c) {
  constexpr int W = 8 * NT;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    red[g * W + nt * 8 + 2 * c] = acc[nt][0];
    red[g * W + nt * 8 + 2 * c + 1] = acc[nt][1];
    red[(g + 8) * W + nt * 8 + 2 * c] = acc[nt][2];
    red[(g + 8) * W + nt * 8 + 2 * c + 1] = acc[nt][3];
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// v0: one thread per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_row_scalar(GemvParams p) {
  write_stamp(0);
  pdl_wait();
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= p.M) return;
  const int groups = p.K >> 7;
  const uint32_t* rw = p.packed + (size_t)row * (p.K >> 3);
  const __half* rs = p.scales + (size_t)row * groups;
  for (int b = 0; b < p.B; ++b) {
    const __half* xb = p.x + (size_t)b * p.K;
    float acc = 0.f;
    for (int G = 0; G < groups; ++G) {
      float part = 0.f;
      for (int j = 0; j < kWordsPerGroup; j += 4) {
        const uint4 w4 = *reinterpret_cast<const uint4*>(rw + G * kWordsPerGroup + j);
        const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          uint32_t h[4];
          unpack_q8(wv[t], h);
          part = dot8_f32(h, ldg_keep(xb + G * kGroup + (j + t) * 8), part);
        }
      }
      acc = fmaf(ldg_half(rs + G), part, acc);
    }
    p.y[(size_t)b * p.M + row] = __float2half_rn(acc);
  }
}

// ---------------------------------------------------------------------------
// v1: one warp per row; lane v reads 16 bytes (32 weights) at 16*(v + 32i):
// 512 contiguous bytes per warp load.  Up to 4 batch rows per pass.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void row_partials(const uint32_t* rw, const __half* rs,
                                             const __half* x, int K, int nb, int first,
                                             int stride, float (&acc)[4]) {
  const int nvec = K >> 5;
  for (int v = first; v < nvec; v += stride) {
    const uint4 w4 = ldg_stream(rw + 4 * v);
    const uint32_t wv[4] = {w4.x, w4.y, w4.z, w4.w};
    const float s = ldg_half(rs + (v >> 2));
    uint32_t h[4][4];
#pragma unroll
    for (int t = 0; t < 4; ++t) unpack_q8(wv[t], h[t]);
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) {
      if (bb < nb) {
        const __half* xb = x + (size_t)bb * K + 32 * v;
        float part = 0.f;
#pragma unroll
        for (int t = 0; t < 4; ++t) part = dot8_f32(h[t], ldg_keep(xb + 8 * t), part);
        acc[bb] = fmaf(s, part, acc[bb]);
      }
    }
  }
}

__global__ void __launch_bounds__(128) k_warp_row(GemvParams p) {
  write_stamp(1);
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (row >= p.M) return;
  const int groups = p.K >> 7;
  const uint32_t* rw = p.packed + (size_t)row * (p.K >> 3);
  const __half* rs = p.scales + (size_t)row * groups;
  for (int b0 = 0; b0 < p.B; b0 += 4) {
    const int nb = min(4, p.B - b0);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    row_partials(rw, rs, p.x + (size_t)b0 * p.K, p.K, nb, lane, 32, acc);
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) {
      const float s = warp_sum(acc[bb]);
      if (lane == 0 && bb < nb) p.y[(size_t)(b0 + bb) * p.M + row] = __float2half_rn(s);
    }
  }
}

// v1 with warps_per_row in [2, 8]: one block per row, warps split K.
__global__ void __launch_bounds__(256) k_block_row(GemvParams p) {
  const int wpr = blockDim.x >> 5;
  write_stamp(10 + wpr);
  pdl_wait();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int row = blockIdx.x;
  const int groups = p.K >> 7;
  const uint32_t* rw = p.packed + (size_t)row * (p.K >> 3);
  const __half* rs = p.scales + (size_t)row * groups;
  __shared__ float red[8][4];
  for (int b0 = 0; b0 < p.B; b0 += 4) {
    const int nb = min(4, p.B - b0);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    row_partials(rw, rs, p.x + (size_t)b0 * p.K, p.K, nb, warp * 32 + lane, wpr * 32, acc);
#pragma unroll
    for (int bb = 0; bb < 4; ++bb) {
      const float s = warp_sum(acc[bb]);
      if (lane == 0) red[warp][bb] = s;
    }
    __syncthreads();
    if (threadIdx.x < nb) {
      float s = 0.f;
      for (int w = 0; w < wpr; ++w) s += red[w][threadIdx.x];
      p.y[(size_t)(b0 + threadIdx.x) * p.M + row] = __float2half_rn(s);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// v2 / v3 / v4: one 16-row tile per CTA (blockIdx.x), 8 warps splitting the
// tile's groups round-robin, 4 groups of 128-bit weight loads in flight per
// warp.  v4 additionally splits the groups over gridDim.y.
// ---------------------------------------------------------------------------
enum TileMode { kTileDirect = 0, kTileScales = 1, kTileSplitK = 2 };
constexpr int kTileWarps = 8;
constexpr int kTilePrefetch = 4;

// Split-K finish: every CTA has stored its groups' products a_G in the
// workspace ([groups][B][M] fp32); the last CTA of the tile to arrive replays
// the canonical order over all groups, so y is bit-identical to v2/v3/v5 for
// any split count.
__device__ __forceinline__ void split_k_finish(const GemvParams& p, int rows, int trow,
                                               unsigned* s_last) {
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) *s_last = atomicAdd(&p.counters[blockIdx.x], 1u);
  __syncthreads();
  if (*s_last != gridDim.y - 1) return;
  __threadfence();
  const int groups = p.K >> 7;
  for (int o = threadIdx.x; o < 16 * p.B; o += blockDim.x) {
    const int r = o % 16, b = o / 16;
    if (r >= rows) continue;
    const float* a = p.ws + (size_t)b * p.M + trow + r;
    const size_t gstride = (size_t)p.B * p.M;
    float y = 0.f;
    for (int w = 0; w < kTileWarps; ++w) {
      float acc = 0.f;
      for (int G = w; G < groups; G += kTileWarps) acc = __fadd_rn(acc, __ldcg(a + G * gstride));
      y = __fadd_rn(y, acc);
    }
    p.y[(size_t)b * p.M + trow + r] = __float2half_rn(y);
  }
  if (threadIdx.x == 0) p.counters[blockIdx.x] = 0u;  // ready for the next call
}

// Stores a_G = scale * D_G of one group for this thread's rows and columns.
template <int NT>
__device__ __forceinline__ void store_group_products(const GemvParams& p, const float (&d)[NT][4],
                                                     float sa, float sb, int G, int trow, int rows,
                                                     int g, int c) {
  float* base = p.ws + (size_t)G * p.B * p.M + trow;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = (j < 2) ? g : g + 8;
      const int b = nt * 8 + 2 * c + (j & 1);
      if (r < rows && b < p.B) base[(size_t)b * p.M + r] = __fmul_rn(j < 2 ? sa : sb, d[nt][j]);
    }
  }
}

template <int NT, int MODE>
__global__ void __launch_bounds__(kTileWarps * 32) k_tile(GemvParams p) {
  write_stamp(MODE == kTileDirect ? 2 : MODE == kTileScales ? 3 : 4);
  constexpr int W = 8 * NT;
  __shared__ float red[kTileWarps][16 * W];
  extern __shared__ __half s_scales[];  // kTileScales: [16][groups in range]
  __shared__ unsigned s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int trow = blockIdx.x * 16;
  const int rows = min(16, p.M - trow);
  const int groups = p.K >> 7;
  int g0 = 0, g1 = groups;
  if (MODE == kTileSplitK) {
    const int per = (groups + gridDim.y - 1) / gridDim.y;
    g0 = min(groups, (int)blockIdx.y * per);
    g1 = min(groups, g0 + per);
  }
  // Rows past M read row rows-1 again; their results are never stored.
  const int ra = trow + min(g, rows - 1), rb = trow + min(g + 8, rows - 1);
  const size_t words = (size_t)(p.K >> 3);
  const uint32_t* wa_ptr = p.packed + (size_t)ra * words + 4 * c;
  const uint32_t* wb_ptr = p.packed + (size_t)rb * words + 4 * c;
  const __half* sa_ptr = p.scales + (size_t)ra * groups;
  const __half* sb_ptr = p.scales + (size_t)rb * groups;

  // Weights are never written by a predecessor kernel (the PDL contract), so
  // their first loads are issued before the dependency wait.
  uint4 wa[kTilePrefetch], wb[kTilePrefetch];
#pragma unroll
  for (int i = 0; i < kTilePrefetch; ++i) {
    const int G = g0 + warp + i * kTileWarps;
    if (G < g1) {
      wa[i] = ldg_stream(wa_ptr + G * kWordsPerGroup);
      wb[i] = ldg_stream(wb_ptr + G * kWordsPerGroup);
    }
  }
  pdl_wait();
  if (MODE == kTileScales) {
    const int ng = g1 - g0;
    for (int i = threadIdx.x; i < 16 * ng; i += blockDim.x) {
      const int r = i / ng, G = g0 + i % ng;
      s_scales[i] = p.scales[(size_t)(trow + min(r, rows - 1)) * groups + G];
    }
    __syncthreads();
  }

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

  for (int base = g0 + warp; base < g1; base += kTilePrefetch * kTileWarps) {
#pragma unroll
    for (int i = 0; i < kTilePrefetch; ++i) {
      const int G = base + i * kTileWarps;
      if (G < g1) {
        const uint4 ca = wa[i], cb = wb[i];
        const int Gn = G + kTilePrefetch * kTileWarps;
        if (Gn < g1) {
          wa[i] = ldg_stream(wa_ptr + Gn * kWordsPerGroup);
          wb[i] = ldg_stream(wb_ptr + Gn * kWordsPerGroup);
        }
        uint4 xr[NT][4];
        load_x_group<NT>(p.x, p.K, p.B, G * kGroup + 32 * c, g, xr);
        float sa, sb;
        if (MODE == kTileScales) {
          const int ng = g1 - g0;
          sa = __half2float(s_scales[g * ng + (G - g0)]);
          sb = __half2float(s_scales[(g + 8) * ng + (G - g0)]);
        } else {
          sa = ldg_half(sa_ptr + G);
          sb = ldg_half(sb_ptr + G);
        }
        float d[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) d[nt][0] = d[nt][1] = d[nt][2] = d[nt][3] = 0.f;
        group_mma<NT>(ca, cb, xr, d);
        if (MODE == kTileSplitK && gridDim.y > 1)
          store_group_products<NT>(p, d, sa, sb, G, trow, rows, g, c);
        else
          scale_accumulate<NT>(acc, d, sa, sb);
      }
    }
  }

  if (MODE == kTileSplitK && gridDim.y > 1) {
    split_k_finish(p, rows, trow, &s_last);
    return;
  }
  store_fragment<NT>(red[warp], acc, g, c);
  __syncthreads();
  for (int o = threadIdx.x; o < 16 * W; o += blockDim.x) {
    const int r = o / W, b = o % W;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kTileWarps; ++w) s = __fadd_rn(s, red[w][o]);
    if (r < rows && b < p.B) p.y[(size_t)b * p.M + trow + r] = __float2half_rn(s);
  }
}


// ---------------------------------------------------------------------------
// v5: persistent bulk-copy pipeline.
//
// CTA i owns rows [i*M/P, (i+1)*M/P): one contiguous span of packed bytes.
// It walks that span as stages of (16-row tile) x (2048-k chunk).  A stage is
// up to 16 row pieces of 1 KB, each one cp.async.bulk issued by its own lane
// of the producer warp into a padded slot (row stride 1088 B, so rows g and
// g+1 fall on opposite halves of the 32 banks and the consumers' 128-bit
// shared loads are conflict-free).  6 slots keep ~100 KB in flight per SM,
// which covers HBM latency x bandwidth / 148 SMs with room to spare.
// ---------------------------------------------------------------------------
namespace v5 {
constexpr int kChunkK = 2048;
constexpr int kChunkGroups = kChunkK / kGroup;  // 16
constexpr int kRowBytes = kChunkK / 2;          // 1024
constexpr int kRowStride = kRowBytes + 64;      // 1088
constexpr int kStageBytes = 16 * kRowStride;    // 17408
constexpr int kStages = 6;
constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
}  // namespace v5

template <int NT>
struct StreamSmem {
  alignas(128) uint8_t stage[v5::kStages][v5::kStageBytes];
  float red[2][v5::kConsumerWarps][16 * 8 * NT];
  uint64_t full[v5::kStages];
  uint64_t empty[v5::kStages];
  int abort_flag;
};

template <int NT, int STAMP>
__global__ void __launch_bounds__(v5::kThreads, 1) k_stream(GemvParams p) {
  using namespace v5;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  StreamSmem<NT>& sm = *reinterpret_cast<StreamSmem<NT>*>(smem_raw);
  write_stamp(STAMP);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = (int)(((long long)blockIdx.x * p.M) / gridDim.x);
  const int r1 = (int)(((long long)(blockIdx.x + 1) * p.M) / gridDim.x);
  const int ntiles = (r1 - r0 + 15) / 16;
  const int groups = p.K / kGroup;
  const int nk = (groups + kChunkGroups - 1) / kChunkGroups;
  const int total = ntiles * nk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    sm.abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  // A dependent GEMV launched with PDL may now start streaming its weights.
  pdl_trigger();
  volatile int* abort_flag = &sm.abort_flag;

  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    const uint64_t policy = policy_evict_first();
    const uint8_t* wbytes = reinterpret_cast<const uint8_t*>(p.packed);
    const size_t row_bytes = (size_t)p.K / 2;
    int issued = 0;
    for (int s = 0; s < total; ++s) {
      const int slot = s % kStages;
      if (s >= kStages && !mbar_wait_bounded(&sm.empty[slot], ((s / kStages) - 1) & 1, abort_flag))
        break;
      const int tile = s / nk, chunk = s % nk;
      const int trow = r0 + tile * 16;
      const int rows = min(16, r1 - trow);
      const uint32_t bytes = (uint32_t)min(kChunkGroups, groups - chunk * kChunkGroups) * 64u;
      if (lane == 0) mbar_arrive_expect_tx(&sm.full[slot], bytes * (uint32_t)rows);
      __syncwarp();
      if (lane < rows) {
        bulk_g2s(smem_u32(sm.stage[slot]) + lane * kRowStride,
                 wbytes + (size_t)(trow + lane) * row_bytes + (size_t)chunk * kRowBytes, bytes,
                 &sm.full[slot], policy);
      }
      issued = s + 1;
    }
    if (*abort_flag && lane == 0) {
      // Let copies already in flight land before the CTA's shared memory is
      // released (bounded as well, against a fresh clock).
      volatile int no_abort = 0;
      for (int s = max(0, issued - kStages); s < issued; ++s)
        mbar_wait_bounded(&sm.full[s % kStages], (s / kStages) & 1, &no_abort);
    }
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();  // x and y belong to the predecessor until here
  const int g = lane >> 2, c = lane & 3;
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;

  for (int s = 0; s < total; ++s) {
    const int slot = s % kStages;
    const int tile = s / nk, chunk = s % nk;
    const int trow = r0 + tile * 16;
    const int rows = min(16, r1 - trow);
    const int cg = min(kChunkGroups, groups - chunk * kChunkGroups);

    // x for this warp's first group of the stage, before waiting on the data.
    uint4 xr[NT][4];
    if (warp < cg) load_x_group<NT>(p.x, p.K, p.B, (chunk * kChunkGroups + warp) * kGroup + 32 * c, g, xr);

    if (mbar_wait_bounded(&sm.full[slot], (s / kStages) & 1, abort_flag)) {
      const uint32_t st = smem_u32(sm.stage[slot]);
      const __half* sa_ptr = p.scales + (size_t)(trow + min(g, rows - 1)) * groups;
      const __half* sb_ptr = p.scales + (size_t)(trow + min(g + 8, rows - 1)) * groups;
      for (int gi = warp; gi < cg; gi += kConsumerWarps) {
        const int G = chunk * kChunkGroups + gi;
        const uint4 wa = lds128(st + g * kRowStride + gi * 64 + c * 16);
        const uint4 wb = lds128(st + (g + 8) * kRowStride + gi * 64 + c * 16);
        const float sa = ldg_half(sa_ptr + G);
        const float sb = ldg_half(sb_ptr + G);
        float d[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) d[nt][0] = d[nt][1] = d[nt][2] = d[nt][3] = 0.f;
        if constexpr (NT == 1) {
          // Double-buffer x: the next group's loads overlap this group's math.
          uint4 xc[NT][4];
#pragma unroll
          for (int t = 0; t < 4; ++t) xc[0][t] = xr[0][t];
          if (gi + kConsumerWarps < cg)
            load_x_group<NT>(p.x, p.K, p.B, (G + kConsumerWarps) * kGroup + 32 * c, g, xr);
          group_mma<NT>(wa, wb, xc, d);
        } else {
          if (gi != warp) load_x_group<NT>(p.x, p.K, p.B, G * kGroup + 32 * c, g, xr);
          group_mma<NT>(wa, wb, xr, d);
        }
        scale_accumulate<NT>(acc, d, sa, sb);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[slot]);

    if (chunk == nk - 1) {
      // Tile complete: sum the consumer warps' partials in warp order.
      float* red = sm.red[tile & 1][0];
      store_fragment<NT>(sm.red[tile & 1][warp], acc, g, c);
      named_barrier(1, kConsumerWarps * 32);
      constexpr int W = 8 * NT;
      for (int o = threadIdx.x; o < 16 * W; o += kConsumerWarps * 32) {
        const int r = o / W, b = o % W;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) sum = __fadd_rn(sum, red[w * 16 * W + o]);
        if (r < rows && b < p.B && !*abort_flag)
          p.y[(size_t)b * p.M + trow + r] = __float2half_rn(sum);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

constexpr int kStampReuse = 15;
constexpr int kMaxBatchPerPass = 32;  // 4 mma n-tiles

template <typename Kern>
dk_status launch(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                 bool pdl, const GemvParams& p, const char* name) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
  if (e != cudaSuccess) {
    set_cuda_error(e, name);
    return DK_ERR_LAUNCH;
  }
  return DK_OK;
}

// Opts a kernel into more than 48 KB of dynamic shared memory, once per device.
template <typename Kern>
dk_status ensure_smem(Kern kernel, size_t bytes, std::atomic<unsigned long long>& done) {
  const int dev = current_device();
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return DK_OK;
  const cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) {
    set_cuda_error(e, "cudaFuncSetAttribute");
    return DK_ERR_CUDA;
  }
  done.fetch_or(bit, std::memory_order_acq_rel);
  return DK_OK;
}

template <int NT, int STAMP>
dk_status launch_stream(const GemvParams& p, cudaStream_t st, bool pdl) {
  static std::atomic<unsigned long long> smem_done{0};
  const size_t smem = sizeof(StreamSmem<NT>);
  dk_status s = ensure_smem(k_stream<NT, STAMP>, smem, smem_done);
  if (s != DK_OK) return s;
  const int grid = std::max(1, std::min(sm_count(-1), (p.M + 7) / 8));
  return launch(k_stream<NT, STAMP>, dim3(grid), dim3(v5::kThreads), smem, st, pdl, p,
                "k_stream");
}

template <int NT, int MODE>
dk_status launch_tile(const GemvParams& p, int split, cudaStream_t st, bool pdl) {
  const int tiles = (p.M + 15) / 16;
  const int groups = p.K / kGroup;
  size_t smem = 0;
  if (MODE == kTileScales) {
    smem = (size_t)16 * groups * sizeof(__half);
    static std::atomic<unsigned long long> smem_done{0};
    if (smem > 48 * 1024) {
      dk_status s = ensure_smem(k_tile<NT, MODE>, smem, smem_done);
      if (s != DK_OK) return s;
    }
  }
  return launch(k_tile<NT, MODE>, dim3(tiles, MODE == kTileSplitK ? split : 1),
                dim3(kTileWarps * 32), smem, st, pdl, p, "k_tile");
}

template <int MODE>
dk_status launch_tile_nt(const GemvParams& p, int split, cudaStream_t st, bool pdl) {
  if (p.B <= 8) return launch_tile<1, MODE>(p, split, st, pdl);
  if (p.B <= 16) return launch_tile<2, MODE>(p, split, st, pdl);
  return launch_tile<4, MODE>(p, split, st, pdl);
}

template <int STAMP>
dk_status launch_stream_nt(const GemvParams& p, cudaStream_t st, bool pdl) {
  if (p.B <= 8) return launch_stream<1, STAMP>(p, st, pdl);
  if (p.B <= 16) return launch_stream<2, STAMP>(p, st, pdl);
  return launch_stream<4, STAMP>(p, st, pdl);
}

// v4 workspace: one arrival counter per 16-row tile (padded to 256 B), then
// the per-group products a_G, fp32 [K/128][B][M], for a pass of up to
// kSplitKBatch batch rows.
constexpr int kSplitKBatch = 8;

size_t splitk_counter_bytes(int M) {
  return ((size_t)(M + 15) / 16 * sizeof(unsigned) + 255) / 256 * 256;
}

size_t splitk_workspace(int M, int K, int B, int split) {
  if (split <= 1) return 0;
  return splitk_counter_bytes(M) +
         (size_t)(K / kGroup) * (size_t)std::min(B, kSplitKBatch) * (size_t)M * sizeof(float);
}

}  // namespace dk

// ===========================================================================
// C ABI
// ===========================================================================
using namespace dk;

extern "C" void dk_gemv_config_init(dk_gemv_config* cfg) {
  if (!cfg) return;
  cfg->version = 5;
  cfg->split_k = 4;
  cfg->reuse_weights = 0;
  cfg->warps_per_row = 1;
  cfg->flags = 0;
}

static dk_status validate_config(const dk_gemv_config& c) {
  // bindings.cpp:41-48
  if (c.version < 0 || c.version > 5) return DK_ERR_INVALID_ARG;
  if (c.split_k < 1 || c.split_k > 32) return DK_ERR_INVALID_ARG;
  if (c.warps_per_row < 1 || c.warps_per_row > 8) return DK_ERR_INVALID_ARG;
  if (c.warps_per_row > 1 && (c.version != 1 || c.reuse_weights)) return DK_ERR_INVALID_ARG;
  if (c.flags & ~DK_FLAG_PDL) return DK_ERR_INVALID_ARG;
  return DK_OK;
}

static int effective_split(int K, const dk_gemv_config& c) {
  if (c.reuse_weights || c.version != 4) return 1;
  return std::max(1, std::min(c.split_k, K / DK_GROUP_SIZE));
}

extern "C" size_t dk_w4a16_workspace_bytes(int M, int K, int B, const dk_gemv_config* cfg) {
  dk_gemv_config c;
  dk_gemv_config_init(&c);
  if (cfg) c = *cfg;
  if (M <= 0 || K <= 0 || B <= 0 || validate_config(c) != DK_OK) return 0;
  return splitk_workspace(M, K, B, effective_split(K, c));
}

extern "C" dk_status dk_w4a16_gemv(const int32_t* packed, const uint16_t* scales,
                                   const uint16_t* x, uint16_t* y, int M, int K, int B,
                                   const dk_gemv_config* cfg, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  dk_gemv_config c;
  dk_gemv_config_init(&c);
  if (cfg) c = *cfg;
  dk_status s = validate_config(c);
  if (s != DK_OK) return s;
  if (M < 0 || K < 0 || B < 0 || K % DK_GROUP_SIZE != 0) return DK_ERR_INVALID_ARG;
  if (M == 0 || B == 0) return DK_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!y) return DK_ERR_INVALID_ARG;
  if (K == 0) {  // empty reduction: y = 0
    const cudaError_t e = cudaMemsetAsync(y, 0, (size_t)B * M * sizeof(uint16_t), st);
    if (e != cudaSuccess) {
      set_cuda_error(e, "cudaMemsetAsync");
      return DK_ERR_CUDA;
    }
    return DK_OK;
  }
  if (!packed || !scales || !x) return DK_ERR_INVALID_ARG;
  if (!aligned16(packed) || !aligned16(x) || (reinterpret_cast<uintptr_t>(scales) & 1u) ||
      (reinterpret_cast<uintptr_t>(y) & 1u))
    return DK_ERR_INVALID_ARG;

  const bool pdl = (c.flags & DK_FLAG_PDL) != 0;
  const int split = effective_split(K, c);
  unsigned* counters = nullptr;
  float* partials = nullptr;
  if (split > 1) {
    const size_t need = splitk_workspace(M, K, B, split);
    if (!workspace || workspace_bytes < need) return DK_ERR_WORKSPACE;
    counters = static_cast<unsigned*>(workspace);
    const size_t cbytes = splitk_counter_bytes(M);
    partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + cbytes);
    const cudaError_t e = cudaMemsetAsync(counters, 0, cbytes, st);
    if (e != cudaSuccess) {
      set_cuda_error(e, "cudaMemsetAsync");
      return DK_ERR_CUDA;
    }
  }

  // Batch rows go through in passes of up to 32 (the kernels' mma n-tiles);
  // v0 and v1 take any B in one launch.
  const bool chunked = c.reuse_weights || c.version >= 2;
  const int step = split > 1 ? kSplitKBatch : chunked ? kMaxBatchPerPass : B;
  for (int b0 = 0; b0 < B; b0 += step) {
    GemvParams p;
    p.packed = reinterpret_cast<const uint32_t*>(packed);
    p.scales = reinterpret_cast<const __half*>(scales);
    p.x = reinterpret_cast<const __half*>(x) + (size_t)b0 * K;
    p.y = reinterpret_cast<__half*>(y) + (size_t)b0 * M;
    p.M = M;
    p.K = K;
    p.B = std::min(step, B - b0);
    p.ws = partials;
    p.counters = counters;
    if (c.reuse_weights) {
      s = launch_stream_nt<kStampReuse>(p, st, pdl);
    } else {
      switch (c.version) {
        case 0:
          s = launch(k_row_scalar, dim3((M + 255) / 256), dim3(256), 0, st, pdl, p,
                     "k_row_scalar");
          break;
        case 1:
          if (c.warps_per_row > 1) {
            const int wpr = std::max(2, std::min(c.warps_per_row, 8));
            s = launch(k_block_row, dim3(M), dim3(wpr * 32), 0, st, pdl, p, "k_block_row");
          } else {
            s = launch(k_warp_row, dim3((M + 3) / 4), dim3(128), 0, st, pdl, p, "k_warp_row");
          }
          break;
        case 2:
          s = launch_tile_nt<kTileDirect>(p, 1, st, pdl);
          break;
        case 3:
          s = launch_tile_nt<kTileScales>(p, 1, st, pdl);
          break;
        case 4:
          s = launch_tile_nt<kTileSplitK>(p, split, st, pdl);
          break;
        default:
          s = launch_stream_nt<5>(p, st, pdl);
          break;
      }
    }
    if (s != DK_OK) return s;
  }
  return DK_OK;
}

extern "C" int dk_last_kernel_stamp(int device) {
  int prev = -1;
  cudaGetDevice(&prev);
  if (device >= 0 && device != prev) cudaSetDevice(device);
  int h = -1;
  cudaDeviceSynchronize();
  if (cudaMemcpyFromSymbol(&h, g_dk_kernel_stamp, sizeof(int)) != cudaSuccess) h = -1;
  if (device >= 0 && device != prev) cudaSetDevice(prev);
  return h;
}

extern "C" int dk_device_error(int device, int clear) {
  int prev = -1;
  cudaGetDevice(&prev);
  if (device >= 0 && device != prev) cudaSetDevice(device);
  int h = -1;
  cudaDeviceSynchronize();
  if (cudaMemcpyFromSymbol(&h, g_dk_device_error, sizeof(int)) != cudaSuccess) h = -1;
  if (clear) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_dk_device_error, &zero, sizeof(int));
  }
  if (device >= 0 && device != prev) cudaSetDevice(prev);
  return h;
}
