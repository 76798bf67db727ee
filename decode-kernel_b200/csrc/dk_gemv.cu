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
//                       the CTA's row block through a shared-memory ring, one
//                       tensor-map TMA box (16 rows x 2 KB, 128-byte swizzle)
//                       per stage plus the stage's scales by cp.async, all
//                       completing on one mbarrier; 16 consumer warps unpack
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
#include <type_traits>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>

#include <cuda.h>
#include <cudaTypedefs.h>

#define DK_DEVICE_GLOBALS
#include "dk_device.cuh"
#include "dk_host.h"


namespace dk {

// Where v5 puts y (the other versions write fp16 y only).
enum OutMode : int {
  kOutHalf = 0,      // fp16 y [B, M]
  kOutFloat = 1,     // fp32 dst[0] [B, M]
  kOutRowShard = 2,  // fp16 into every rank's dst[g] [B, ld] at columns col0 + m
  kOutKShard = 3,    // fp32 partial into every rank's dst[g] [world][B][M], slot `rank`, as
                     // 64-bit {value, call number} words (low-latency exchange)
  kOutRowGather = 4, // row shard, low-latency exchange: every rank's dst[g] [B, ld] of 64-bit
                     // {fp16-rounded value as fp32, call number} words at columns col0 + m
                     // (the K-shard words' format); the kernel then gathers the whole
                     // [B, ld] of fp16 into y (GemvParams::y)
};
constexpr int kMaxShards = DK_MAX_SHARDS;
struct OutSpec {
  int mode = kOutHalf;
  int world = 1, rank = 0;
  int ld = 0, col0 = 0;
  void* dst[kMaxShards] = {};
  unsigned* slots[kMaxShards] = {};  // shard modes: each rank's arrival slots
  unsigned* seq = nullptr;           // shard modes: this rank's [calls done, grid]
  int grid = 0;                      // shard modes: CTAs per rank (same on every rank)
  int await_all = 0;                 // row shards: CTA 0 waits for every rank's part;
                                     // K shards: the kernel sums the world's partials
                                     // of its rows into fp16 y (GemvParams::y)
};

// v5 row segments: several weight matrices sharing x, run as one GEMV over
// their concatenated rows (q/k/v, gate/up).  Segment s owns the global 16-row
// tiles [tile0, tile0 + ceil(rows / 16)); its last tile may be partial.
constexpr int kMaxSeg = DK_MAX_SEGMENTS;
struct Segment {
  const uint32_t* packed;  // [rows, K/8]
  const __half* scales;    // [rows, K/128]
  __half* y;               // [B, rows]
  int rows, tile0;
};
// Paired (gate/up SiLU-mul) mode: n == 2 with equal rows; the tiles run as
// (gate tile j, up tile j) pairs, CTAs own whole pairs, and only s[0].y --
// h = silu(gate) * up -- is written.
struct SegList {
  int n;       // 2..kMaxSeg
  int paired;  // 1: gate/up SiLU-mul pairs
  Segment s[kMaxSeg];
  __host__ __device__ int pairs() const { return (s[0].rows + 15) / 16; }
  __host__ __device__ int tiles() const {
    return paired ? 2 * pairs() : s[n - 1].tile0 + (s[n - 1].rows + 15) / 16;
  }
  // Units the CTAs split: pairs, or tiles.
  __host__ __device__ int units() const { return paired ? pairs() : tiles(); }
};

struct GemvParams {
  const uint32_t* packed;  // [M, K/8]
  const __half* scales;    // [M, K/128]
  const __half* x;         // [B, ldx]
  __half* y;               // [B, M]
  int M, K, B;
  int ldx;                 // row stride of x in elements (K, or more for a K slice)
  float* ws;               // v4: [K/128][B][M] fp32 per-group products
  unsigned* counters;      // v4: one arrival counter per 16-row tile
  int stages;              // v5: ring depth
  int xs_bytes;            // v5: bytes of x staged in shared memory (0 = none)
  int red_bufs;            // v5: tile-sum buffers (2 or 4)
  OutSpec out;             // v5: destination of y
};

// A CTA's share of a v5 call: whole 16-row tiles, so no CTA fetches or
// computes rows of its neighbour.  One matrix: tiles [t0, t0 + ntiles) =
// [bid·T/grid, (bid+1)·T/grid) of the T = ceil(M/16) tiles, rows [r0, r1)
// (only the matrix's last tile may be partial).  Several matrices: whole
// global tiles [t0, t0 + ntiles) of the segments' concatenation, each inside
// one segment.
struct TileRef {
  int seg, row, rows;  // segment, first row inside it, valid rows
};
// Segment modes of the v5 kernel (compile-time, so the single-matrix kernel
// carries no segment code): one matrix, several, gate/up SiLU-mul pairs.
constexpr int kSegOne = 0, kSegMulti = 1, kSegPair = 2;

// v5 kernel argument besides GemvParams: the weights' tensor maps and, for
// several matrices, their segments (kept out of GemvParams: a larger
// GemvParams measurably slows the single-matrix kernel).
template <bool MULTI>
struct StreamArgs {
  CUtensorMap m[1];
};
template <>
struct StreamArgs<true> {
  CUtensorMap m[kMaxSeg];
  SegList segs;
};

template <int SEG>
struct CtaTiles {
  static constexpr bool MULTI = SEG != kSegOne;
  int r0, r1;     // one matrix
  int t0;         // several matrices
  int ntiles;
  __device__ __forceinline__ void init(const GemvParams& p, const StreamArgs<MULTI>& a) {
    if constexpr (!MULTI) {
      const int T = (p.M + 15) / 16;
      t0 = (int)(((long long)blockIdx.x * T) / gridDim.x);
      ntiles = (int)(((long long)(blockIdx.x + 1) * T) / gridDim.x) - t0;
      r0 = t0 * 16;
      r1 = min(p.M, (t0 + ntiles) * 16);
    } else {
      const int ntot = a.segs.units();
      t0 = (int)(((long long)blockIdx.x * ntot) / gridDim.x);
      ntiles = (int)(((long long)(blockIdx.x + 1) * ntot) / gridDim.x) - t0;
      if constexpr (SEG == kSegPair) {
        t0 *= 2;
        ntiles *= 2;
      }
      r0 = r1 = 0;
    }
  }
  __device__ __forceinline__ TileRef operator()(const StreamArgs<MULTI>& a, int t) const {
    if constexpr (!MULTI) {
      const int row = r0 + t * 16;
      return {0, row, min(16, r1 - row)};
    } else {
      const int gt = t0 + t;
      if constexpr (SEG == kSegPair) {
        const int row = (gt >> 1) * 16;
        return {gt & 1, row, min(16, a.segs.s[0].rows - row)};
      }
      int s = 0;
      while (s + 1 < a.segs.n && gt >= a.segs.s[s + 1].tile0) ++s;
      const int row = (gt - a.segs.s[s].tile0) * 16;
      return {s, row, min(16, a.segs.s[s].rows - row)};
    }
  }
};

// v5 result store for batch row b, output row m.  `tag`: the call's sequence
// number (K-shard mode only).
// GATHER: the kernel compiles the row-gather words (one n-tile kernels only: the
// code costs the 2- and 4-n-tile kernels registers they do not have).
template <bool GATHER>
__device__ __forceinline__ void store_y(const GemvParams& p, int b, int m, float v,
                                        unsigned tag = 0) {
  switch (p.out.mode) {
    case kOutFloat:
      static_cast<float*>(p.out.dst[0])[(size_t)b * p.M + m] = v;
      break;
    case kOutRowShard: {
      const __half h = __float2half_rn(v);
      for (int g = 0; g < p.out.world; ++g)
        static_cast<__half*>(p.out.dst[g])[(size_t)b * p.out.ld + p.out.col0 + m] = h;
      break;
    }
    case kOutKShard:
      for (int g = 0; g < p.out.world; ++g)
        st_ll_sys(static_cast<unsigned long long*>(p.out.dst[g]) +
                      ((size_t)p.out.rank * p.B + b) * p.M + m,
                  v, tag);
      break;
    case kOutRowGather:
      if constexpr (GATHER) {
        const float h = __half2float(__float2half_rn(v));  // fp16 -> fp32 -> fp16 is exact
        for (int g = 0; g < p.out.world; ++g)
          st_ll_sys(static_cast<unsigned long long*>(p.out.dst[g]) + (size_t)b * p.out.ld +
                        p.out.col0 + m,
                    h, tag);
      }
      break;
    default:
      p.y[(size_t)b * p.M + m] = __float2half_rn(v);
  }
}

// Shard modes: after this CTA's last store of y, mark its arrival slot in
// every rank's slot array with the call's sequence number (release stores at
// system scope: the warp's stores to that rank are visible before the mark).
// With await_all CTA 0 then waits (bounded) until every slot of this rank's
// own array carries the number, so the kernel -- and the stream -- completes
// with the gather complete while a PDL-launched successor already streams
// its weights.  Called by the one warp that wrote y, all lanes.
__device__ __forceinline__ void signal_shards(const GemvParams& p, int lane) {
  if (p.out.mode != kOutRowShard) return;  // K-shard words carry their own call number
  pdl_wait();  // seq was advanced by the previous sharded call
  const unsigned epoch = *reinterpret_cast<volatile unsigned*>(p.out.seq) + 1;
  __syncwarp();
  if (lane < p.out.world)
    st_release_sys(p.out.slots[lane] + p.out.rank * DK_SHARD_SLOTS + blockIdx.x, epoch);
  if (blockIdx.x != 0) return;
  if (p.out.await_all) {
    wait_slots(p.out.slots[p.out.rank], DK_SHARD_SLOTS, p.out.world, (int)gridDim.x, epoch,
               &g_dk_device_error);
    if (lane == 0) p.out.seq[0] = epoch;
  }
  if (lane == 0) p.out.seq[1] = gridDim.x;
}

// K-shard mode with the sum fused (ranks on separate GPUs, running at once):
// after this CTA has stored its partials of all its tiles into every rank's
// buffer, it polls this rank's buffer for every rank's word of the same rows
// -- the same CTA of every rank owns the same rows -- until each carries this
// call's number, adds the ranks in order (0 + p_0 + p_1 + ..., the
// arithmetic of dk_shard_reduce, so the same bits) and stores fp16 y.  The
// CTA that finishes last advances the call number (seq[0]; seq[2] counts the
// CTAs), as the separate sum's last block does.  Bounded: 2 s after the first
// poll it records kDevWaitTimeout and stops.  Called by the tile-sum warp,
// all lanes.
template <class Args, class Tiles>
__device__ __forceinline__ void sum_kshards(const GemvParams& p, const Args& a, const Tiles& tiles,
                                            int ntiles, int nb, unsigned tag, int lane,
                                            volatile int* abort_flag) {
  const unsigned long long* part =
      static_cast<const unsigned long long*>(p.out.dst[p.out.rank]);
  const size_t rank_stride = (size_t)p.B * p.M;
  const int world = p.out.world;
  // One pass over all of this CTA's (row, batch column) outputs, 32 at a
  // time.  Each lane first loads every rank's word of its output -- the
  // loads are independent, so they are in flight together -- and then polls
  // again only the words that do not carry this call's number yet: the wait
  // costs about one L2 round trip per pass, not one per rank and tile.
  const int per_tile = 16 * nb;
  const int total = ntiles * per_tile;
  const uint64_t t0 = globaltimer_ns();
  bool timed_out = false;
  for (int o0 = 0; o0 < total && !timed_out; o0 += 32) {
    const int o = o0 + lane;
    const int t = o / per_tile, q = o - t * per_tile, r = q / nb, b = q - r * nb;
    bool live = o < total;
    size_t i = 0;
    if (live) {
      const TileRef tr = tiles(a, t);
      live = r < tr.rows;
      i = (size_t)b * p.M + tr.row + r;
    }
    if (live) {
      unsigned long long w[kMaxShards];
#pragma unroll
      for (int g = 0; g < kMaxShards; ++g)
        if (g < world) w[g] = ld_ll_sys(part + g * rank_stride + i);
      float sum = 0.f;
#pragma unroll
      for (int g = 0; g < kMaxShards; ++g) {
        if (g >= world) break;
        for (unsigned polls = 1; (unsigned)(w[g] >> 32) != tag && !timed_out; ++polls) {
          if ((polls & 255u) == 0 && (*abort_flag || globaltimer_ns() - t0 > kWaitLimitNs)) {
            if (!*abort_flag) atomicExch(&g_dk_device_error, kDevWaitTimeout);
            *abort_flag = 1;
            timed_out = true;
          } else {
            w[g] = ld_ll_sys(part + g * rank_stride + i);
          }
        }
        sum = __fadd_rn(sum, __uint_as_float((unsigned)w[g]));
      }
      if (!timed_out) p.y[i] = __float2half_rn(sum);
    }
    timed_out = __any_sync(0xffffffffu, timed_out);
  }
  __syncwarp();
  if (lane == 0) {
    if (atomicAdd(p.out.seq + 2, 1u) == gridDim.x - 1) {
      p.out.seq[2] = 0;
      p.out.seq[0] = tag;
    }
  }
}

// Row shards with the gather fused (ranks on separate GPUs, running at once):
// after this CTA has stored its rows into every rank's buffer as 64-bit
// {value, call number} words, it takes its share [bid·ld/grid, (bid+1)·ld/grid)
// of the full gathered width, polls this rank's buffer until each of those
// words carries this call's number (whichever rank wrote it), and stores the
// fp16 values into y [B, ld].  The words carry their own call number -- the
// full 32 bits, so no stale word of another layer's exchange in the same
// buffer set can pass for this call's -- and neither a fence behind the stores
// nor an arrival handshake is needed.  The CTA that finishes last advances the
// call number (seq[0]; seq[2] counts the CTAs).  Bounded like sum_kshards.
// Called by the tile-sum warp, all lanes.
__device__ __forceinline__ void gather_rows(const GemvParams& p, unsigned tag, int lane,
                                            volatile int* abort_flag) {
  const unsigned long long* words = static_cast<const unsigned long long*>(p.out.dst[p.out.rank]);
  const int ld = p.out.ld;
  const int g0 = (int)((long long)blockIdx.x * ld / gridDim.x);
  const int g1 = (int)((long long)(blockIdx.x + 1) * ld / gridDim.x);
  const int n = g1 - g0;
  // kU words per lane per pass: loaded together, then polled again only
  // where they do not carry this call's number yet.
  constexpr int kU = 4;
  const uint64_t t0 = globaltimer_ns();
  bool timed_out = false;
  for (int o0 = 0; o0 < n * p.B && !timed_out; o0 += 32 * kU) {
    unsigned long long w[kU];
    long long idx[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int o = o0 + u * 32 + lane;
      idx[u] = -1;
      if (o < n * p.B) {
        const int b = o / n, m = g0 + (o - b * n);
        idx[u] = (long long)b * ld + m;
        w[u] = ld_ll_sys(words + idx[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (idx[u] < 0) continue;
      for (unsigned polls = 1; (unsigned)(w[u] >> 32) != tag && !timed_out; ++polls) {
        if ((polls & 255u) == 0 && (*abort_flag || globaltimer_ns() - t0 > kWaitLimitNs)) {
          if (!*abort_flag) atomicExch(&g_dk_device_error, kDevWaitTimeout);
          *abort_flag = 1;
          timed_out = true;
        } else {
          w[u] = ld_ll_sys(words + idx[u]);
        }
      }
      if (!timed_out) p.y[idx[u]] = __float2half_rn(__uint_as_float((unsigned)w[u]));
    }
    timed_out = __any_sync(0xffffffffu, timed_out);
  }
  __syncwarp();
  if (lane == 0) {
    if (atomicAdd(p.out.seq + 2, 1u) == gridDim.x - 1) {
      p.out.seq[2] = 0;
      p.out.seq[0] = tag;
    }
  }
}

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
// x[nt*8 + g][kx + 8t .. kx + 8t + 7], t = 0..3, kx = 128*G + 32*c.  Lanes
// whose batch column is past B read row B-1 instead: mma columns are
// independent and those columns are never stored.
template <int NT>
__device__ __forceinline__ void load_x_group(const __half* __restrict__ x, int K, int B, int kx,
                                             int g, uint4 (&xr)[NT][4]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const __half* xb = x + (size_t)min(nt * 8 + g, B - 1) * K + kx;
#pragma unroll
    for (int t = 0; t < 4; ++t) xr[nt][t] = ldg_keep(xb + 8 * t);
  }
}

// One group (128 k) of a 16-row tile: thread (g, c) holds words 4c..4c+3 of
// the group for rows g (wa) and g+8 (wb).  Eight HMMAs; the quad's four
// threads supply the 16 k of each one, all inside this group, so the group
// scale can be applied to the fp32 result afterwards.  The eight run as one
// accumulation chain from zero, word t = 0..3 in order and each word's two
// MMAs in order: that chain is D_G, and every kernel computes it this way.
// (Two chains joined by an add cost one more fp32 add per output per group;
// ILP comes from the independent groups and warps instead.)
__device__ __forceinline__ void word_mma(float (&d)[4], uint32_t wa, uint32_t wb,
                                         const uint32_t (&px)[4]) {
  uint32_t ha[4], hb[4];
  unpack_q8(wa, ha);
  unpack_q8(wb, hb);
  mma16816(d, ha[0], hb[0], ha[1], hb[1], px[0], px[1]);
  mma16816(d, ha[2], hb[2], ha[3], hb[3], px[2], px[3]);
}

template <int NT>
__device__ __forceinline__ void group_mma(const uint4& wa, const uint4& wb,
                                          const uint4 (&xr)[NT][4], float (&d)[NT][4]) {
  const uint32_t A[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t Bw[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      uint32_t px[4];
      pair_x8(xr[nt][t], px);
      word_mma(d[nt], A[t], Bw[t], px);
    }
  }
}

// Canonical reduction order, shared by v2, v3, v4, v5 and the reuse path so
// that all of them return the same bits for the same inputs (and y[b] does
// not depend on which other batch rows or output rows are in the call):
//   acc_w    = fma(s_G, D_G, acc_w) for G = w, w+16, w+32, ... (from 0),
//              w = 0..15; s_G = scale[m, G] in fp32, D_G the group's HMMA
//              chain; one fp32 rounding per group (fused multiply-add)
//   y        = fp16_rn((((0 + acc_0) + acc_1) + ...) + acc_15)
// fmaf is always fused and the sums use _rn intrinsics, so the compiler can
// neither split the one nor contract the other.
constexpr int kClasses = 16;

template <int NT>
__device__ __forceinline__ void scale_accumulate(float (&acc)[NT][4], const float (&d)[NT][4],
                                                 float sa, float sb) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    acc[nt][0] = fmaf(sa, d[nt][0], acc[nt][0]);
    acc[nt][1] = fmaf(sa, d[nt][1], acc[nt][1]);
    acc[nt][2] = fmaf(sb, d[nt][2], acc[nt][2]);
    acc[nt][3] = fmaf(sb, d[nt][3], acc[nt][3]);
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

// Split-K finish: every CTA has stored its groups' HMMA chains D_G in the
// workspace ([groups][B][M] fp32); the last CTA of the tile to arrive replays
// the canonical order over all groups with the scales, so y is bit-identical
// to v2/v3/v5 for any split count.
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
    const float* dg = p.ws + (size_t)b * p.M + trow + r;
    const __half* sg = p.scales + (size_t)(trow + r) * groups;
    const size_t gstride = (size_t)p.B * p.M;
    float y = 0.f;
    for (int w = 0; w < kClasses; ++w) {
      float acc = 0.f;
      for (int G = w; G < groups; G += kClasses)
        acc = fmaf(ldg_half(sg + G), __ldcg(dg + G * gstride), acc);
      y = __fadd_rn(y, acc);
    }
    p.y[(size_t)b * p.M + trow + r] = __float2half_rn(y);
  }
  if (threadIdx.x == 0) p.counters[blockIdx.x] = 0u;  // ready for the next call
}

// Stores D_G, one group's HMMA chain, for this thread's rows and columns.
template <int NT>
__device__ __forceinline__ void store_group_products(const GemvParams& p, const float (&d)[NT][4],
                                                     int G, int trow, int rows, int g, int c) {
  float* base = p.ws + (size_t)G * p.B * p.M + trow;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = (j < 2) ? g : g + 8;
      const int b = nt * 8 + 2 * c + (j & 1);
      if (r < rows && b < p.B) base[(size_t)b * p.M + r] = d[nt][j];
    }
  }
}

template <int NT, int MODE>
__global__ void __launch_bounds__(kTileWarps * 32) k_tile(GemvParams p) {
  write_stamp(MODE == kTileDirect ? 2 : MODE == kTileScales ? 3 : 4);
  constexpr int W = 8 * NT;
  __shared__ float red[kClasses][16 * W];
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

  // Warp w covers groups G = w (mod 8), i.e. classes w and w + 8 of the
  // canonical order; acc[j] holds the class reached on the j-th parity step.
  float acc[2][NT][4];
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      acc[j][nt][0] = acc[j][nt][1] = acc[j][nt][2] = acc[j][nt][3] = 0.f;
  const int cls0 = ((g0 + warp) >> 3) & 1;  // class bit of this warp's first group

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
          store_group_products<NT>(p, d, G, trow, rows, g, c);
        else
          scale_accumulate<NT>(acc[i & 1], d, sa, sb);
      }
    }
  }

  if (MODE == kTileSplitK && gridDim.y > 1) {
    split_k_finish(p, rows, trow, &s_last);
    return;
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) store_fragment<NT>(red[warp + 8 * ((cls0 + j) & 1)], acc[j], g, c);
  __syncthreads();
  for (int o = threadIdx.x; o < 16 * W; o += blockDim.x) {
    const int r = o / W, b = o % W;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kClasses; ++w) s = __fadd_rn(s, red[w][o]);
    if (r < rows && b < p.B) p.y[(size_t)b * p.M + trow + r] = __float2half_rn(s);
  }
}


// ---------------------------------------------------------------------------
// v5: persistent TMA pipeline.
//
// CTA i owns rows [i*M/P, (i+1)*M/P).  It walks them as stages of (16-row
// tile) x (4096-k chunk): 16 rows x 2 KB of packed weights.  When K is a
// multiple of 256 the producer fetches a stage with ONE tensor-map TMA copy
// (a 3-D view of the weights: 128-byte strips x rows x strips, 128-byte
// swizzle) and the stage's 16 x 32 scales with 4-byte cp.async, all
// completing on the stage's mbarrier; otherwise it issues one 1-D bulk copy
// per row into rows padded to 2112 bytes and the consumers read the scales
// from global memory one stage ahead.  Few, large copy operations matter on
// B200: with ~100 KB in flight per SM, 1 KB copies stream at ~2.2 TB/s while
// 16-32 KB tensor boxes reach ~5 TB/s.
//
// Bank conflicts: under the 128-byte swizzle, 16-byte chunk j of tile row r
// sits at chunk position j ^ (r & 7).  A quarter-warp of the consumers' 128-bit
// fragment loads covers two mma rows; mapping mma row g to tile row
// {0,4,1,5,2,6,3,7}[g] (and g+8 to 8 + that) puts those two rows on opposite
// halves of the banks, so every fragment load is conflict-free.  (The padded
// bulk layout is conflict-free with the identity mapping.)
//
// Activations: when the pass's x rows fit in kXsMaxBytes -- or, on the 16-warp
// kernel, in what is left beside a 2-stage ring and 2 tile-sum buffers (x up to
// ~130 KB: K = 8192 at 8 rows) -- the consumers load
// them once (after the PDL wait -- x may be the previous kernel's output) and
// store every 128-k group rearranged so that a group's B fragments are four
// conflict-free 128-bit loads: the pairs of word t for quad lane c sit at
// 16 * (4t + c); each batch row is padded by 64 bytes.  Larger x is read from
// global memory per group.  Batch lanes past B read batch row B-1 (their
// columns are discarded).
//
// Tile results: every consumer warp stores its partial sums and moves on; the
// producer warp, which polls instead of blocking, adds the 16 classes in order
// and writes y -- kRedBufs buffers guarded by mbarriers, no CTA-wide barrier.
// ---------------------------------------------------------------------------
namespace v5 {
constexpr int kChunkK = 4096;                   // k per stage
constexpr int kChunkGroups = kChunkK / kGroup;  // 32
constexpr int kRowBytes = kChunkK / 2;          // 2048 bytes of a row per stage
constexpr int kPadRowStride = kRowBytes + 64;   // 2112 (bulk path)
constexpr int kStageBytesBulk = 16 * kPadRowStride;    // 33792
constexpr int kStageBytesTma = 16 * kRowBytes;         // 32768
constexpr int kScaleRowStride = kChunkGroups * 2 + 4;  // 68: rows land on distinct banks
constexpr int kStageScaleBytes = 16 * kScaleRowStride;  // 1088 (TMA path)
constexpr int kStrip = 128;                             // bytes per swizzle strip
constexpr int kStripsPerChunk = kRowBytes / kStrip;     // 16
constexpr int kMaxStages = 6;
constexpr int kMinStages = 2;
constexpr int kStagesBeforeX = 2;  // weight stages issued before x is staged
// Consumer warps: 16 (one CTA per SM, deepest ring) or 8 (a CTA small enough
// that two fit on an SM, so a GEMV launched behind this one with PDL streams
// its weights while this one computes).  Warp w handles groups w, w + NCW, ...
// of every stage; group gi is class gi mod 16 of the canonical order, so with
// 16 warps warp w owns class w and with 8 warps classes w and w + 8.
template <int NCW>
struct Consumers {
  static constexpr int kWarps = NCW;
  static constexpr int kThreads = NCW * 32;
  static constexpr int kGroupsPerWarp = kChunkGroups / NCW;   // 2 or 4
  static constexpr int kClassesPerWarp = kClasses / NCW;       // 1 or 2
};
constexpr int kXsMaxBytes = 68 * 1024;
constexpr int kSmemCap = 227 * 1024;  // per-CTA opt-in maximum on sm_100
// Shared-memory budget per CTA: the whole SM for 16 warps, half of it (minus
// the per-CTA reserve) for 8 warps.
__host__ __device__ constexpr int smem_budget(int ncw) { return ncw == 16 ? 220 * 1024 : 110 * 1024; }

__host__ __device__ constexpr int stage_bytes(bool tmap) {
  return tmap ? kStageBytesTma : kStageBytesBulk;
}
__host__ __device__ inline int xs_row_stride(int K) { return 2 * K + 64; }

struct Layout {
  int sc_off, xs_off, red_off, bar_off, total;
};

// Tile partial sums: kRedBufs buffers of [class][tile row][red_cols] floats,
// so a consumer warp reaching the end of a tile never waits for the producer
// to have added up the tile before last.  One n-tile keeps only the batch
// columns that exist (rounded up to the even pair a quad lane stores).
constexpr int kRedBufs = 4;     // at most; GemvParams::red_bufs is the launch's count
constexpr int kMinRedBufs = 2;  // (a launch uses 2 or 4: the ring index is a mask)
__host__ __device__ inline int red_cols(int nt, int B) { return nt == 1 ? ((B + 1) & ~1) : 8 * nt; }

__host__ __device__ inline Layout layout(int nt, bool tmap, int stages, int xs_bytes, int nbp,
                                         int red_bufs = kRedBufs) {
  Layout L;
  int off = stages * stage_bytes(tmap);
  L.sc_off = off;
  off += tmap ? (stages * kStageScaleBytes + 127) / 128 * 128 : 0;
  L.xs_off = off;
  off += (xs_bytes + 127) / 128 * 128;
  L.red_off = off;
  off += red_bufs * kClasses * 16 * nbp * (int)sizeof(float);
  L.bar_off = off;
  off += (2 * kMaxStages + 2 * kRedBufs + 1) * 8 + 16;  // full, empty, red_full, red_free, xready, flag
  L.total = off;
  return L;
}
}  // namespace v5

// Stage walker: (tile, chunk) in tile-major order plus the ring slot/round,
// advanced without divisions.
struct StageCursor {
  int tile = 0, chunk = 0, slot = 0, round = 0;
  __device__ __forceinline__ void next(int nk, int stages) {
    if (++chunk == nk) {
      chunk = 0;
      ++tile;
    }
    if (++slot == stages) {
      slot = 0;
      ++round;
    }
  }
};

// Tile row that mma row r (0..15) reads.
template <bool TMAP>
__device__ __forceinline__ int tile_row(int r) {
  if constexpr (TMAP) return (r & 8) | ((r & 1) << 2) | ((r >> 1) & 3);
  return r;
}

// Offset inside a stage of quad lane c's 16 bytes of group gi in tile row R.
template <bool TMAP>
__device__ __forceinline__ uint32_t frag_off(int R, int gi, int c) {
  if constexpr (TMAP) {
    const int j = ((gi & 1) << 2) | c;  // 16-byte chunk inside the 128-byte strip
    return (gi >> 1) * (16 * v5::kStrip) + R * v5::kStrip + ((j ^ (R & 7)) << 4);
  }
  return R * v5::kPadRowStride + gi * 64 + c * 16;
}

// One group, B fragments from the rearranged shared copy of x (same chain as
// group_mma).
__device__ __forceinline__ void group_mma_xs(const uint4& wa, const uint4& wb, uint32_t xq,
                                             float (&d)[4]) {
  const uint32_t A[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t Bw[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint4 x4 = lds128(xq + 64 * t);
    const uint32_t px[4] = {x4.x, x4.y, x4.z, x4.w};
    word_mma(d, A[t], Bw[t], px);
  }
}

// One group with x read from global memory, for the streaming kernel: the
// weights are unpacked once and reused for every n-tile, and x is loaded one
// n-tile at a time (register budget at 544 threads).  Same HMMA chain as
// group_mma, so the same bits.
template <int NT>
__device__ __forceinline__ void group_mma_gx(const uint4& wa, const uint4& wb,
                                             const __half* __restrict__ x, int K, int B, int kx,
                                             int g, float (&d)[NT][4]) {
  const uint32_t A[4] = {wa.x, wa.y, wa.z, wa.w};
  const uint32_t Bw[4] = {wb.x, wb.y, wb.z, wb.w};
  uint32_t ha[4][4], hb[4][4];
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    unpack_q8(A[t], ha[t]);
    unpack_q8(Bw[t], hb[t]);
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const __half* xb = x + (size_t)min(nt * 8 + g, B - 1) * K + kx;
    uint4 xr[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) xr[t] = ldg_keep(xb + 8 * t);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      uint32_t px[4];
      pair_x8(xr[t], px);
      mma16816(d[nt], ha[t][0], hb[t][0], ha[t][1], hb[t][1], px[0], px[1]);
      mma16816(d[nt], ha[t][2], hb[t][2], ha[t][3], hb[t][3], px[2], px[3]);
    }
  }
}


template <int NT, int STAMP, bool XS, bool TMAP, int NCW, int SEG>
__global__ void __launch_bounds__(NCW * 32 + 64, NCW == 8 ? 2 : 1)
    k_stream(const __grid_constant__ StreamArgs<SEG != kSegOne> a, GemvParams p) {
  using namespace v5;
  constexpr bool MULTI = SEG != kSegOne;
  using CW = Consumers<NCW>;
  constexpr int kConsumerWarps = CW::kWarps;
  constexpr int kConsumerThreads = CW::kThreads;
  constexpr int kGroupsPerWarp = CW::kGroupsPerWarp;
  constexpr int kAcc = CW::kClassesPerWarp;
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int kStageBytes = stage_bytes(TMAP);
  constexpr int W = 8 * NT;  // mma output columns per tile row
  const int stages = p.stages;
  const int nbp = red_cols(NT, p.B);
  // Tile-sum buffers in use, 2 or 4: ring slot t & (n - 1), round t >> (n / 2).
  // Only the 16-warp one-n-tile kernel with x staged ever runs with 2 (the
  // largest staged x); every other kernel keeps the count a constant (a
  // runtime count costs the 2- and 4-n-tile kernels spills).
  constexpr bool kRuntimeRed = NCW == 16 && NT == 1 && XS;
  const int nred = kRuntimeRed ? p.red_bufs : kRedBufs, rmask = nred - 1, rshift = nred >> 1;
  const Layout L = layout(NT, TMAP, stages, XS ? p.xs_bytes : 0, nbp, nred);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* empty = full + kMaxStages;
  uint64_t* red_full = empty + kMaxStages;    // [kRedBufs]: all consumer warps stored a tile
  uint64_t* red_free = red_full + kRedBufs;   // [kRedBufs]: the producer has read it
  uint64_t* xready = red_free + kRedBufs;     // the consumers have staged x
  volatile int* abort_flag = reinterpret_cast<volatile int*>(xready + 1);
  float* red = reinterpret_cast<float*>(smem + L.red_off);
  const uint32_t ring = smem_u32(smem);
  const uint32_t scs = smem_u32(smem + L.sc_off);
  const uint32_t xs = smem_u32(smem + L.xs_off);
  write_stamp(STAMP);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  CtaTiles<SEG> tiles;
  tiles.init(p, a);
  const int ntiles = tiles.ntiles;
  const int groups = p.K / kGroup;
  const int nk = (groups + kChunkGroups - 1) / kChunkGroups;
  const int total = ntiles * nk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      // TMA path: the box's transaction bytes (1 arrival) plus one cp.async
      // arrival per producer lane for the stage's scales.
      mbar_init(&full[s], TMAP ? 33 : 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int i = 0; i < kRedBufs; ++i) {
      mbar_init(&red_full[i], kConsumerWarps);
      mbar_init(&red_free[i], 1);
    }
    mbar_init(xready, 1);
    *abort_flag = 0;
    fence_barrier_init();
    if constexpr (TMAP) {
      if constexpr (MULTI) {
        for (int i = 0; i < a.segs.n; ++i) tma_prefetch_desc(&a.m[i]);
      } else {
        tma_prefetch_desc(&a.m[0]);
      }
    }
  }
  __syncthreads();
  // A dependent GEMV launched with PDL may now start streaming its weights.
  pdl_trigger();

  if (warp == kConsumerWarps) {
    // ---------------- issuer: weight stages ----------------
    // It only issues copies, so it waits in bounded blocking waits (a warp
    // suspended in try_wait takes no issue slots from the consumer warps that
    // share its sub-partition; a slot comes back only once every consumer warp
    // has released it, so a starved warp would pace the whole CTA).
    const uint64_t policy = policy_evict_first();
    const size_t row_bytes = (size_t)p.K / 2;
    StageCursor cur;
    int issued = 0;
    for (; issued < total; ++issued) {
      // x is loaded by the consumers while the first stages stream; holding
      // the rest back until it has landed keeps those loads from queueing
      // behind a full ring of weight copies.
      if (XS && issued == kStagesBeforeX && !mbar_wait_bounded(xready, 0, abort_flag)) break;
      if (issued >= stages &&
          !mbar_wait_bounded(&empty[cur.slot], (cur.round - 1) & 1, abort_flag))
        break;
      const TileRef tr = tiles(a, cur.tile);
      const CUtensorMap* tmap;
      const __half* sscales;
      const uint32_t* spacked;
      if constexpr (MULTI) {
        tmap = &a.m[tr.seg];
        sscales = a.segs.s[tr.seg].scales;
        spacked = a.segs.s[tr.seg].packed;
      } else {
        tmap = &a.m[0];
        sscales = p.scales;
        spacked = p.packed;
      }
      const int trow = tr.row;
      const uint32_t dst = ring + cur.slot * kStageBytes;
      if constexpr (TMAP) {
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[cur.slot], (uint32_t)kStageBytes);
          tma_load_3d(dst, tmap, 0, trow, cur.chunk * kStripsPerChunk, &full[cur.slot], policy);
        }
        // Scales of the stage: 16 rows x 32 groups, 4 bytes (2 groups) per
        // cp.async.  K % 256 == 0 here, so scale rows are 4-byte aligned.
        // Rows past the matrix are not loaded (their weights arrive
        // zero-filled and their results are never stored).
        const uint32_t sdst = scs + cur.slot * kStageScaleBytes;
        const int gbase = cur.chunk * kChunkGroups;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int i = lane + 32 * k, r = i >> 4, w2 = (i & 15) * 2;
          if (r < tr.rows && gbase + w2 < groups)
            cp_async4(sdst + r * kScaleRowStride + w2 * 2,
                      sscales + (size_t)(trow + r) * groups + gbase + w2);
        }
        cp_async_mbar_arrive(&full[cur.slot]);
      } else {
        const int rows = tr.rows;
        const uint32_t bytes =
            (uint32_t)min(kChunkGroups, groups - cur.chunk * kChunkGroups) * 64u;
        if (lane == 0) mbar_arrive_expect_tx(&full[cur.slot], bytes * (uint32_t)rows);
        __syncwarp();
        if (lane < rows) {
          const uint8_t* wbytes = reinterpret_cast<const uint8_t*>(spacked);
          bulk_g2s(dst + lane * kPadRowStride,
                   wbytes + (size_t)(trow + lane) * row_bytes + (size_t)cur.chunk * kRowBytes,
                   bytes, &full[cur.slot], policy);
        }
      }
      cur.next(nk, stages);
    }
    // Stay until the copies issued last have landed: if another warp aborts,
    // the consumers leave without waiting for them, and the CTA's shared
    // memory must outlive every copy into it (bounded as well, against a
    // fresh clock, and regardless of the abort flag).
    if (lane == 0) {
      volatile int no_abort = 0;
      for (int s2 = max(0, issued - stages); s2 < issued; ++s2)
        mbar_wait_bounded(&full[s2 % stages], (s2 / stages) & 1, &no_abort);
    }
    return;
  }

  if (warp == kConsumerWarps + 1) {
    // ---------------- reducer: tile sums ----------------
    // Tile t: the 16 class partials of every real row and batch column, added
    // in class order.  It waits suspended on earlier tiles (their sums are off
    // the critical path) and polls for the CTA's last one, whose sum and
    // store end the kernel.
    const int nb = min(W, p.B);
    // Word-exchange modes: this call's number (the previous call advanced
    // it).  One n-tile reads it while the consumers stage x, off the path
    // from the first tile's partials to its stores; the wider kernels read it
    // at their first tile (earlier costs them registers).
    unsigned tag = 0;
    if constexpr (!MULTI && NT == 1) {
      if (p.out.mode == kOutKShard || p.out.mode == kOutRowGather) {
        pdl_wait();
        tag = *reinterpret_cast<volatile const unsigned*>(p.out.seq) + 1;
      }
    }
    for (int t = 0; t < ntiles; ++t) {
      uint64_t* bar = &red_full[t & rmask];
      const uint32_t par = (t >> rshift) & 1;
      const bool ok = t + 1 < ntiles ? mbar_wait_bounded(bar, par, abort_flag)
                                     : mbar_wait_poll_bounded(bar, par, abort_flag);
      if (!ok) return;
      const float* rt = red + (t & rmask) * kClasses * 16 * nbp;
      const TileRef tr = tiles(a, t);
      const int trow = tr.row, rows = tr.rows;
      if (!MULTI && NT != 1 && t == 0 && p.out.mode == kOutKShard) {
        pdl_wait();  // the number was advanced by the previous call's sum
        tag = *reinterpret_cast<volatile const unsigned*>(p.out.seq) + 1;
      }
      constexpr bool paired = SEG == kSegPair;
      if (paired && tr.seg == 0) continue;  // gate tile: kept until its up tile
      for (int o = lane; o < rows * nb; o += 32) {
        const int r = o / nb, b = o - r * nb;
        const float* src = rt + r * nbp + b;
        float sum = 0.f;
#pragma unroll
        for (int w = 0; w < kClasses; ++w) sum = __fadd_rn(sum, src[w * 16 * nbp]);
        if constexpr (MULTI) {
          if (paired) {
            // h = silu(g) * u with the roundings of the unfused fp16
            // sequence: g and u as GEMV outputs, silu(g) = g / (1 +
            // exp(-g)) in fp32 rounded to fp16, the product in fp32
            // rounded to fp16.
            const float* gsrc = red + ((t - 1) & rmask) * kClasses * 16 * nbp + r * nbp + b;
            float gsum = 0.f;
#pragma unroll
            for (int w = 0; w < kClasses; ++w) gsum = __fadd_rn(gsum, gsrc[w * 16 * nbp]);
            const float gv = __half2float(__float2half_rn(gsum));
            const float sg = __half2float(__float2half_rn(gv / (1.0f + expf(-gv))));
            const float u = __half2float(__float2half_rn(sum));
            const Segment& s0 = a.segs.s[0];
            s0.y[(size_t)b * s0.rows + trow + r] = __float2half_rn(__fmul_rn(sg, u));
          } else {
            const Segment& sg = a.segs.s[tr.seg];
            sg.y[(size_t)b * sg.rows + trow + r] = __float2half_rn(sum);
          }
        } else {
          store_y<!MULTI && NT == 1>(p, b, trow + r, sum, tag);
        }
      }
      __syncwarp();
      if (lane == 0) {
        if (paired) mbar_arrive(&red_free[(t - 1) & rmask]);
        mbar_arrive(&red_free[t & rmask]);
      }
    }
    // (one n-tile only: the code would cost the 2- and 4-n-tile kernels registers;
    // larger batches take the separate sum, dk_w4a16_gemv_kshard_sum)
    if constexpr (!MULTI && NT == 1) {
      const bool ksum = p.out.mode == kOutKShard && p.out.await_all;
      const bool gather = p.out.mode == kOutRowGather;
      // (a CTA without rows takes part too: it counts itself in)
      if (ksum) sum_kshards(p, a, tiles, ntiles, nb, tag, lane, abort_flag);
      if (gather) gather_rows(p, tag, lane, abort_flag);
    }
    signal_shards(p, lane);
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();  // x and y belong to the predecessor until here
  const int g = lane >> 2, c = lane & 3;
  const int ra = tile_row<TMAP>(g), rb = tile_row<TMAP>(g + 8);  // this lane's tile rows
  const int bb = min(g, p.B - 1);  // batch row this lane feeds into the mma
  const int xrow = xs_row_stride(p.K);
  if (XS) {
    // Stage x: raw 16-byte chunk i of a row holds k = 8i..8i+7, i.e. word
    // t = i % 4 of quad lane c = (i / 4) % 4 of group i / 16; it is stored,
    // as pairs (x0,x4),(x1,x5),(x2,x6),(x3,x7), at chunk 4t + c of its
    // group.  Loads go through L2 only (x may have just been written by the
    // predecessor grid; no L1 line from an earlier kernel is trusted).
    // With more than two chunks per thread, the thread's chunks j = tid,
    // tid + T, ... of the flattened [B, K/8] array are loaded kXLoads at a
    // time before any of them is stored: the shared store is a compiler
    // barrier, so in a load-store loop no load can be issued before the
    // previous chunk's store, and the issuer holds the weight stream back
    // until x has landed (4096^2, B = 8: 7.95 -> 6.85 us).  With one or two
    // chunks (B = 1 up to K = 4096 on 8 warps) the plain per-row loop
    // measured faster (3.93 against 4.19 us at 4096^2).
    constexpr int kXLoads = 8;
    const int cpr = p.K / 8;
    if (p.B * cpr <= 2 * kConsumerThreads) {
      for (int b = 0; b < p.B; ++b) {
        const uint4* src = reinterpret_cast<const uint4*>(p.x + (size_t)b * p.ldx);
        const uint32_t rowbase = xs + (uint32_t)(b * xrow);
#pragma unroll 2
        for (int i = threadIdx.x; i < cpr; i += kConsumerThreads) {
          uint32_t pr[4];
          pair_x8(ldcg128(src + i), pr);
          const int ii = i & 15;
          sts128(rowbase + (uint32_t)(i >> 4) * 256u + 16u * (4 * (ii & 3) + (ii >> 2)), pr);
        }
      }
    } else {
      int b = 0, i = threadIdx.x;
      while (i >= cpr) i -= cpr, ++b;
      while (b < p.B) {
        uint4 v[kXLoads];
        uint32_t dst[kXLoads];
#pragma unroll
        for (int u = 0; u < kXLoads; ++u) {
          dst[u] = 0xffffffffu;
          if (b < p.B) {
            v[u] = ldcg128(reinterpret_cast<const uint4*>(p.x + (size_t)b * p.ldx) + i);
            const int ii = i & 15;
            dst[u] = xs + (uint32_t)(b * xrow) + (uint32_t)(i >> 4) * 256u +
                     16u * (4 * (ii & 3) + (ii >> 2));
            for (i += kConsumerThreads; i >= cpr; i -= cpr) ++b;
          }
        }
#pragma unroll
        for (int u = 0; u < kXLoads; ++u) {
          if (dst[u] != 0xffffffffu) {
            uint32_t pr[4];
            pair_x8(v[u], pr);
            sts128(dst[u], pr);
          }
        }
      }
    }
    named_barrier(1, kConsumerThreads);
    if (threadIdx.x == 0) mbar_arrive(xready);
  }

  // Per-thread offsets, fixed for the whole kernel.  Warp w takes groups
  // w + j * NCW (j < kGroupsPerWarp) of every stage; NCW is even, so group j's
  // fragments sit a compile-time stride after group 0's.
  static_assert(NCW % 2 == 0, "fragment strides assume an even warp count");
  constexpr uint32_t kFragStride = TMAP ? (NCW / 2) * 16 * kStrip : NCW * 64;
  const uint32_t offa = frag_off<TMAP>(ra, warp, c), offb = frag_off<TMAP>(rb, warp, c);
  const uint32_t sc_a = ra * kScaleRowStride + warp * 2, sc_b = rb * kScaleRowStride + warp * 2;
  const uint32_t xq = xs + bb * xrow + 16 * c + 256u * warp;  // + 256 (32 chunk + NCW j) + 64 t

  // acc[a]: this warp's class warp + a * NCW.
  float acc[kAcc][NT][4];
#pragma unroll
  for (int a = 0; a < kAcc; ++a)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[a][nt][0] = acc[a][nt][1] = acc[a][nt][2] = acc[a][nt][3] = 0.f;

  // Bulk path: scales from global memory, loaded one stage ahead (sn) and
  // used by the stage after (scur).
  float sn[kGroupsPerWarp][2], scur[kGroupsPerWarp][2];
  auto load_scales = [&](int tile, int chunk) {
    const TileRef tr = tiles(a, tile);
    const __half* sp;
    if constexpr (MULTI) {
      sp = a.segs.s[tr.seg].scales + (size_t)tr.row * groups;
    } else {
      sp = p.scales + (size_t)tr.row * groups;
    }
#pragma unroll
    for (int j = 0; j < kGroupsPerWarp; ++j) {
      const int G = min(chunk * kChunkGroups + warp + j * kConsumerWarps, groups - 1);
      sn[j][0] = ldg_half(sp + (size_t)min(ra, tr.rows - 1) * groups + G);
      sn[j][1] = ldg_half(sp + (size_t)min(rb, tr.rows - 1) * groups + G);
    }
  };
  if (!TMAP && total > 0) load_scales(0, 0);

  // One stage.  Group j's fragments and scales are read from the slot right
  // before its math, and the slot goes back to the producer once the warp's
  // last group has been read; no register copy of the whole stage (the 18- or
  // 20-warp layouts cap a thread at 96 registers: 5 warps share the busiest
  // sub-partition's 16K).  With two n-tiles (9..16 batch rows, x from global
  // memory) the next group's fragments are read during the current group's
  // math instead, which measured faster there (4096^2, B = 16: 10.8 vs
  // 11.7 us) and slower everywhere else.  FULL: all 32 groups of the chunk
  // exist (no per-group guards).
  struct Frag {
    uint4 wa, wb;
    float sa, sb;
  };
  auto stage = [&](auto full, uint32_t st, uint32_t sst, uint64_t* empty_bar, int chunk) {
    constexpr bool FULL = decltype(full)::value;
    const int cg = FULL ? kChunkGroups : groups - chunk * kChunkGroups;
    const uint32_t xc = xq + 256u * kChunkGroups * chunk;
    auto have = [&](int j) { return FULL || warp + j * kConsumerWarps < cg; };
    auto load = [&](int j, Frag& f) {
      f.wa = lds128(st + offa + j * kFragStride);
      f.wb = lds128(st + offb + j * kFragStride);
      if constexpr (TMAP) {
        f.sa = lds_half(sst + sc_a + j * 2 * kConsumerWarps);
        f.sb = lds_half(sst + sc_b + j * 2 * kConsumerWarps);
      } else {
        f.sa = scur[j][0];
        f.sb = scur[j][1];
      }
    };
    auto release = [&]() {
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar);
    };
    auto math = [&](int j, const Frag& f) {
      float d[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) d[nt][0] = d[nt][1] = d[nt][2] = d[nt][3] = 0.f;
      if constexpr (XS) {
        group_mma_xs(f.wa, f.wb, xc + 256u * kConsumerWarps * j, d[0]);
      } else {
        const int G = chunk * kChunkGroups + warp + j * kConsumerWarps;
        group_mma_gx<NT>(f.wa, f.wb, p.x, p.ldx, p.B, G * kGroup + 32 * c, g, d);
      }
      scale_accumulate<NT>(acc[j % kAcc], d, f.sa, f.sb);
    };
    Frag f[2];
    if constexpr (NT != 2) {
#pragma unroll
      for (int j = 0; j < kGroupsPerWarp; ++j) {
        if (have(j)) load(j, f[0]);
        if (j == kGroupsPerWarp - 1) release();
        if (have(j)) math(j, f[0]);
      }
    } else {
      if (have(0)) load(0, f[0]);
      if (kGroupsPerWarp > 1 && have(1)) load(1, f[1]);
      if (kGroupsPerWarp <= 2) release();
#pragma unroll
      for (int j = 0; j < kGroupsPerWarp; ++j) {
        if (have(j)) math(j, f[j & 1]);
        if (j + 2 < kGroupsPerWarp) {
          if (have(j + 2)) load(j + 2, f[j & 1]);
          if (j + 2 == kGroupsPerWarp - 1) release();
        }
      }
    }
  };

  const bool last_chunk_full = groups % kChunkGroups == 0;
  int slot = 0, chunk = 0, tile = 0;
  uint32_t phase = 0;
  for (int s = 0; s < total; ++s) {
    if (!mbar_wait_bounded(&full[slot], phase, abort_flag)) return;  // timed out: abort
    const uint32_t st = ring + slot * kStageBytes;
    const uint32_t sst = scs + slot * kStageScaleBytes;
    const bool last = chunk == nk - 1;
    if constexpr (!TMAP) {
#pragma unroll
      for (int j = 0; j < kGroupsPerWarp; ++j) scur[j][0] = sn[j][0], scur[j][1] = sn[j][1];
      if (s + 1 < total) load_scales(last ? tile + 1 : tile, last ? 0 : chunk + 1);
    }
    if (!last || last_chunk_full) {
      stage(std::true_type{}, st, sst, &empty[slot], chunk);
    } else {
      stage(std::false_type{}, st, sst, &empty[slot], chunk);
    }
    if (++slot == stages) {
      slot = 0;
      phase ^= 1u;
    }
    if (last) {
      // Tile complete: each warp stores its class partials and moves on; the
      // producer warp adds them up.  A buffer is rewritten only after the
      // producer has read the tile red_bufs back.
      chunk = 0;
      const int rs = tile & rmask;
      float* rt = red + rs * kClasses * 16 * nbp;
      if (tile >= nred &&
          !mbar_wait_bounded(&red_free[rs], ((tile >> rshift) - 1) & 1, abort_flag))
        return;
#pragma unroll
      for (int a = 0; a < kAcc; ++a) {
        float* mine = rt + (warp + a * NCW) * 16 * nbp;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (nt * 8 + 2 * c < p.B) {  // columns past B are never read
            mine[ra * nbp + nt * 8 + 2 * c] = acc[a][nt][0];
            mine[ra * nbp + nt * 8 + 2 * c + 1] = acc[a][nt][1];
            mine[rb * nbp + nt * 8 + 2 * c] = acc[a][nt][2];
            mine[rb * nbp + nt * 8 + 2 * c + 1] = acc[a][nt][3];
          }
          acc[a][nt][0] = acc[a][nt][1] = acc[a][nt][2] = acc[a][nt][3] = 0.f;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_full[rs]);
      ++tile;
    } else {
      ++chunk;
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

constexpr int kStampReuse = 15;
constexpr int kMaxBatchPerPass = 32;  // 4 mma n-tiles

// Host half of the dispatch stamp.  The reference clears the device stamp to
// -1 with a copy before every launch (gemv_w4a16.cu:553-557), so a call that
// launches nothing leaves -1 behind.  A copy on the caller's stream would sit
// between two PDL-chained GEMVs and serialise them, so here every GEMV entry
// point marks its device "nothing launched" on entry and "launched" once a
// kernel launch has succeeded; dk_last_kernel_stamp reports -1 while the mark
// says nothing was launched, and the stamp the kernel wrote otherwise.
constexpr int kStampDevices = 64;
std::atomic<int> g_stamp_live[kStampDevices];

void stamp_begin_call() {
  const int dev = current_device();
  if (dev >= 0 && dev < kStampDevices) g_stamp_live[dev].store(0, std::memory_order_relaxed);
}

void stamp_launched() {
  const int dev = current_device();
  if (dev >= 0 && dev < kStampDevices) g_stamp_live[dev].store(1, std::memory_order_relaxed);
}

bool stamp_is_live(int dev) {
  return dev >= 0 && dev < kStampDevices && g_stamp_live[dev].load(std::memory_order_relaxed);
}

template <typename Kern, typename... Args>
dk_status launch(const char* name, Kern kernel, dim3 grid, dim3 block, size_t smem,
                 cudaStream_t stream, bool pdl, Args... args) {
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
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) {
    set_cuda_error(e, name);
    return DK_ERR_LAUNCH;
  }
  stamp_launched();
  return DK_OK;
}

// Opts a kernel into more than 48 KB of dynamic shared memory, once per device.
template <typename Kern>
dk_status ensure_smem(Kern kernel, size_t bytes, std::atomic<unsigned long long>& done) {
  const int dev = current_device();
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return DK_OK;
  cudaError_t e =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  // Without this the driver may size the SM's shared-memory carveout for one
  // small CTA and leave no room for a second resident CTA.
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) {
    set_cuda_error(e, "cudaFuncSetAttribute");
    return DK_ERR_CUDA;
  }
  done.fetch_or(bit, std::memory_order_acq_rel);
  return DK_OK;
}

// Tensor map of the packed weights for the v5 TMA path: a 3-D view
// {128-byte strip, row, strip index} with strides {K/2, 128} bytes, boxes of
// 16 rows x 16 strips (32 KB), 128-byte swizzle.  Encoded once per
// (pointer, M, K) -- the map holds nothing else -- and kept in a small cache.
using EncodeTiledFn = PFN_cuTensorMapEncodeTiled_v12000;

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

bool weight_tensor_map(const void* packed, int M, int K, CUtensorMap* out) {
  struct Entry {
    const void* ptr;
    int M, K;
    unsigned long long stamp;
    CUtensorMap map;
  };
  static std::mutex mu;
  static Entry cache[64];
  static unsigned long long clock = 0;
  std::lock_guard<std::mutex> lk(mu);
  Entry* victim = &cache[0];
  for (Entry& e : cache) {
    if (e.stamp && e.ptr == packed && e.M == M && e.K == K) {
      e.stamp = ++clock;
      *out = e.map;
      return true;
    }
    if (e.stamp < victim->stamp) victim = &e;
  }
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  CUtensorMap map;
  cuuint64_t dims[3] = {(cuuint64_t)v5::kStrip, (cuuint64_t)M, (cuuint64_t)(K / 256)};
  cuuint64_t strides[2] = {(cuuint64_t)K / 2, (cuuint64_t)v5::kStrip};
  cuuint32_t box[3] = {(cuuint32_t)v5::kStrip, 16u, (cuuint32_t)v5::kStripsPerChunk};
  cuuint32_t elem[3] = {1, 1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(packed), dims, strides, box,
          elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  victim->ptr = packed;
  victim->M = M;
  victim->K = K;
  victim->stamp = ++clock;
  victim->map = map;
  *out = map;
  return true;
}

// Per (device, stream): whether the last k_stream launch there ran exactly
// one 8-warp CTA on every SM.  Only then does each SM keep one CTA slot free
// for a PDL-launched successor, so that the successor's CTAs land one per SM;
// after a 16-warp kernel, two CTAs of the same call per SM or a grid smaller
// than the SM count, the SMs that free first can take two of them and finish
// last.  A hint for the next launch's warp count only: a stale or wrong entry
// costs time, never results (every warp count computes the same bits).
class StreamHistory {
 public:
  bool one_per_sm(int device, cudaStream_t st) {
    std::lock_guard<std::mutex> lk(mu_);
    for (const Entry& e : e_)
      if (e.stamp && e.device == device && e.st == st) return e.one_per_sm;
    return false;
  }
  void record(int device, cudaStream_t st, bool one_per_sm) {
    std::lock_guard<std::mutex> lk(mu_);
    Entry* victim = &e_[0];
    for (Entry& e : e_) {
      if (e.stamp && e.device == device && e.st == st) {
        victim = &e;
        break;
      }
      if (e.stamp < victim->stamp) victim = &e;
    }
    *victim = Entry{st, device, one_per_sm, ++clock_};
  }

 private:
  struct Entry {
    cudaStream_t st;
    int device;
    bool one_per_sm;
    unsigned long long stamp;
  };
  std::mutex mu_;
  Entry e_[32] = {};
  unsigned long long clock_ = 0;
};
StreamHistory g_stream_history;

template <int NT, int STAMP, bool XS, bool TMAP, int NCW, int SEG>
dk_status launch_stream_cfg(GemvParams p, const StreamArgs<SEG != kSegOne>& a, cudaStream_t st,
                            bool pdl, int ctas_per_sm = 1) {
  static std::atomic<unsigned long long> smem_done{0};
  p.xs_bytes = XS ? p.B * v5::xs_row_stride(p.K) : 0;
  p.stages = v5::kMaxStages;
  p.red_bufs = v5::kRedBufs;
  auto total = [&]() {
    return v5::layout(NT, TMAP, p.stages, p.xs_bytes, v5::red_cols(NT, p.B), p.red_bufs).total;
  };
  // Ring depth first, then (only for the largest staged x) tile-sum buffers.
  while (p.stages > v5::kMinStages && total() > v5::smem_budget(NCW)) --p.stages;
  if (NCW == 16 && NT == 1 && XS && total() > v5::smem_budget(NCW)) p.red_bufs = v5::kMinRedBufs;
  const size_t smem = total();
  if (smem > (size_t)v5::kSmemCap) return DK_ERR_UNSUPPORTED;
  dk_status s = ensure_smem(k_stream<NT, STAMP, XS, TMAP, NCW, SEG>, v5::kSmemCap, smem_done);
  if (s != DK_OK) return s;
  int units = (p.M + 15) / 16;  // one matrix: its 16-row tiles
  if constexpr (SEG != kSegOne) units = a.segs.units();
  const int sms = sm_count(-1);
  const int grid = p.out.grid > 0 ? p.out.grid : std::max(1, std::min(ctas_per_sm * sms, units));
  s = launch("k_stream", k_stream<NT, STAMP, XS, TMAP, NCW, SEG>, dim3(grid),
             dim3(NCW * 32 + 64), smem, st, pdl, a, p);
  if (s == DK_OK) g_stream_history.record(current_device(), st, NCW == 8 && grid == sms);
  return s;
}

// 8 consumer warps (two CTAs per SM) while a CTA's share of the weights is
// small -- then a CTA's life is dominated by latency and overlapping the next
// GEMV pays most -- and while the 8-warp layout keeps at least 2 stages in
// half of the SM's shared memory; 16 warps otherwise.  A 16-warp CTA shares
// its SM with no other CTA (registers), so a GEMV next to one in a stream
// gets no overlap on either side: in the Llama-2-7B layer sequence the
// 4096x11008 down projection (176 KB per CTA) on 8 warps takes the 32-layer
// step from 1621 to 1263 us although alone it is 4 % slower (8.46 vs 8.15
// us) -- but only behind a launch that left one slot free on every SM
// (StreamHistory): behind the SiLU-mul pair (two CTAs per SM) the same
// projection in the tensor-parallel layer sequence is faster on 16 warps
// (1137 vs 1245 us per 32 layers), and so is the 12288-row q/k/v launch
// (192 KB) behind it (1245 vs 1331).  Shares above 192 KB stay on 16 warps:
// with 8 warps the Llama-3-8B MLP (224-229 KB) made that model's step slower
// (1483 -> 1839 us).
template <int NT, bool XS, bool TMAP>
bool use_coresident(const GemvParams& p, cudaStream_t st) {
#if defined(DK_V5_FORCE_NCW)
  return DK_V5_FORCE_NCW == 8;
#else
  const int tiles = (p.M + 15) / 16;
  const int grid = std::max(1, std::min(sm_count(-1), tiles));
  const size_t cta_bytes = (size_t)((tiles + grid - 1) / grid) * 16 * (size_t)p.K / 2;
  const int xs = XS ? p.B * v5::xs_row_stride(p.K) : 0;
  const size_t limit =
      (cta_bytes > 160 * 1024 && g_stream_history.one_per_sm(current_device(), st) ? 192 : 160) *
      1024;
  return NT == 1 && XS && cta_bytes <= limit &&
         v5::layout(NT, TMAP, v5::kMinStages, xs, v5::red_cols(NT, p.B)).total <=
             v5::smem_budget(8);
#endif
}

// Two 8-warp CTAs of the same call per SM (grid 2 x SMs) on one large
// matrix: each consumer warp then takes 4 groups of a stage instead of 2, so
// the per-stage work (barrier waits, slot release, bookkeeping) is spread
// over twice the weights.  It pays only when every CTA keeps several tiles
// (28672x8192, B=1: 25.4 vs 26.5 us); with 1-2 tiles per CTA the SMs whose
// CTAs differ in tile count idle half their warps (8192x28672: 33.4 vs 27.4).
template <int NT, bool XS, bool TMAP, int SEG>
bool use_two_ctas_per_sm(const GemvParams& p) {
  if (!(NT == 1 && XS && TMAP && (SEG == kSegOne || SEG == kSegPair)) || p.out.grid > 0)
    return false;
  const int tiles = (p.M + 15) / 16;
  const int xs = XS ? p.B * v5::xs_row_stride(p.K) : 0;
  return tiles >= 8 * sm_count(-1) &&
         v5::layout(NT, TMAP, v5::kMinStages, xs, v5::red_cols(NT, p.B)).total <=
             v5::smem_budget(8);
}

template <int NT, int STAMP, bool XS, bool TMAP, int SEG>
dk_status launch_stream_w(const GemvParams& p, const StreamArgs<SEG != kSegOne>& a, cudaStream_t st,
                          bool pdl) {
  if constexpr (NT == 1 && XS) {
    if (use_coresident<NT, XS, TMAP>(p, st))
      return launch_stream_cfg<NT, STAMP, XS, TMAP, 8, SEG>(p, a, st, pdl);
    if (use_two_ctas_per_sm<NT, XS, TMAP, SEG>(p))
      return launch_stream_cfg<NT, STAMP, XS, TMAP, 8, SEG>(p, a, st, pdl, 2);
  }
  return launch_stream_cfg<NT, STAMP, XS, TMAP, 16, SEG>(p, a, st, pdl);
}

#include "dk_batch.cuh"

template <int NT, int STAMP, bool TMAP, int SEG>
dk_status launch_stream_x(const GemvParams& p, const StreamArgs<SEG != kSegOne>& a, cudaStream_t st,
                          bool pdl) {
  const int xs = p.B * v5::xs_row_stride(p.K);
  const bool staged = xs <= v5::kXsMaxBytes || v5::layout(1, TMAP, v5::kMinStages, xs, v5::red_cols(1, p.B), v5::kMinRedBufs).total <= v5::smem_budget(16);
  if (NT == 1 && staged) return launch_stream_w<1, STAMP, true, TMAP, SEG>(p, a, st, pdl);
  return launch_stream_w<NT, STAMP, false, TMAP, SEG>(p, a, st, pdl);
}

// The weights' tensor maps (TMA when every matrix has one; K % 256 keeps a
// stage's 16 KB box whole), then the launch.  A single matrix (segs null)
// runs the kernel compiled without segment indexing.
template <int NT, int STAMP, int SEG>
dk_status launch_stream_a(const GemvParams& p, StreamArgs<SEG != kSegOne>& a, cudaStream_t st,
                          bool pdl) {
  bool tma = p.K % 256 == 0;
  if constexpr (SEG != kSegOne) {
    for (int i = 0; tma && i < a.segs.n; ++i)
      tma = weight_tensor_map(a.segs.s[i].packed, a.segs.s[i].rows, p.K, &a.m[i]);
  } else {
    tma = tma && weight_tensor_map(p.packed, p.M, p.K, &a.m[0]);
  }
  if (tma) return launch_stream_x<NT, STAMP, true, SEG>(p, a, st, pdl);
  std::memset(a.m, 0, sizeof(a.m));
  return launch_stream_x<NT, STAMP, false, SEG>(p, a, st, pdl);
}

template <int NT, int STAMP>
dk_status launch_stream(const GemvParams& p, const SegList* segs, cudaStream_t st, bool pdl) {
  if (segs) {
    StreamArgs<true> a;
    std::memset(&a, 0, sizeof(a));
    a.segs = *segs;
    if (segs->paired) return launch_stream_a<NT, STAMP, kSegPair>(p, a, st, pdl);
    return launch_stream_a<NT, STAMP, kSegMulti>(p, a, st, pdl);
  }
  StreamArgs<false> a;
  std::memset(&a, 0, sizeof(a));
  return launch_stream_a<NT, STAMP, kSegOne>(p, a, st, pdl);
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
  return launch("k_tile", k_tile<NT, MODE>, dim3(tiles, MODE == kTileSplitK ? split : 1),
                dim3(kTileWarps * 32), smem, st, pdl, p);
}

template <int MODE>
dk_status launch_tile_nt(const GemvParams& p, int split, cudaStream_t st, bool pdl) {
  if (p.B <= 8) return launch_tile<1, MODE>(p, split, st, pdl);
  if (p.B <= 16) return launch_tile<2, MODE>(p, split, st, pdl);
  return launch_tile<4, MODE>(p, split, st, pdl);
}

// segs: several matrices sharing x (null: the one matrix of p).
template <int STAMP>
dk_status launch_stream_nt(const GemvParams& p, cudaStream_t st, bool pdl,
                           const SegList* segs = nullptr) {
  if (p.B <= 8) return launch_stream<1, STAMP>(p, segs, st, pdl);
  if (!segs) {
    const dk_status b = launch_batch<STAMP>(p, st, pdl);  // tensor cores, large W, 17..32 rows
    if (b != DK_ERR_UNSUPPORTED) return b;
  }
  if (p.B <= 16) return launch_stream<2, STAMP>(p, segs, st, pdl);
  return launch_stream<4, STAMP>(p, segs, st, pdl);
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
  if (c.flags & ~(DK_FLAG_PDL | DK_FLAG_F32_OUT | DK_FLAG_SHARD_WAIT)) return DK_ERR_INVALID_ARG;
  return DK_OK;
}

// fp32 output exists on the v5 pipeline only.
static bool f32_supported(const dk_gemv_config& c) { return c.reuse_weights || c.version == 5; }

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
  stamp_begin_call();
  dk_gemv_config c;
  dk_gemv_config_init(&c);
  if (cfg) c = *cfg;
  dk_status s = validate_config(c);
  if (s != DK_OK) return s;
  if (M < 0 || K < 0 || B < 0 || K % DK_GROUP_SIZE != 0) return DK_ERR_INVALID_ARG;
  if (M == 0 || B == 0) return DK_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!y) return DK_ERR_INVALID_ARG;
  const bool f32 = (c.flags & DK_FLAG_F32_OUT) != 0;
  if (f32 && !f32_supported(c)) return DK_ERR_UNSUPPORTED;
  if (c.flags & DK_FLAG_SHARD_WAIT) return DK_ERR_INVALID_ARG;  // sharded calls only
  if (K == 0) {  // empty reduction: y = 0
    const size_t elem = f32 ? sizeof(float) : sizeof(uint16_t);
    const cudaError_t e = cudaMemsetAsync(y, 0, (size_t)B * M * elem, st);
    if (e != cudaSuccess) {
      set_cuda_error(e, "cudaMemsetAsync");
      return DK_ERR_CUDA;
    }
    return DK_OK;
  }
  if (!packed || !scales || !x) return DK_ERR_INVALID_ARG;
  if (!aligned16(packed) || !aligned16(x) || (reinterpret_cast<uintptr_t>(scales) & 1u) ||
      (reinterpret_cast<uintptr_t>(y) & (f32 ? 3u : 1u)))
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
    p.ldx = K;
    p.B = std::min(step, B - b0);
    if (f32) {
      p.out.mode = kOutFloat;
      p.out.dst[0] = reinterpret_cast<float*>(y) + (size_t)b0 * M;
    }
    p.ws = partials;
    p.counters = counters;
    if (c.reuse_weights) {
      s = launch_stream_nt<kStampReuse>(p, st, pdl);
    } else {
      switch (c.version) {
        case 0:
          s = launch("k_row_scalar", k_row_scalar, dim3((M + 255) / 256), dim3(256), 0, st, pdl,
                     p);
          break;
        case 1:
          if (c.warps_per_row > 1) {
            const int wpr = std::max(2, std::min(c.warps_per_row, 8));
            s = launch("k_block_row", k_block_row, dim3(M), dim3(wpr * 32), 0, st, pdl, p);
          } else {
            s = launch("k_warp_row", k_warp_row, dim3((M + 3) / 4), dim3(128), 0, st, pdl, p);
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

// ---------------------------------------------------------------------------
// Several weight matrices sharing x in one launch (q/k/v, gate/up): the v5
// pipeline over the concatenation of their row tiles.
// ---------------------------------------------------------------------------
extern "C" dk_status dk_w4a16_gemv_multi(int n, const int32_t* const* packed,
                                         const uint16_t* const* scales, const int* M,
                                         uint16_t* const* y, const uint16_t* x, int K, int B,
                                         const dk_gemv_config* cfg, void* stream) {
  stamp_begin_call();
  dk_gemv_config c;
  dk_gemv_config_init(&c);
  if (cfg) c = *cfg;
  dk_status s = validate_config(c);
  if (s != DK_OK) return s;
  if (c.flags & DK_FLAG_SHARD_WAIT) return DK_ERR_INVALID_ARG;
  if (n < 1 || n > kMaxSeg || !packed || !scales || !M || !y || K < 0 || B < 0 ||
      K % DK_GROUP_SIZE != 0)
    return DK_ERR_INVALID_ARG;
  if ((c.version != 5 && !c.reuse_weights) || (c.flags & DK_FLAG_F32_OUT)) return DK_ERR_UNSUPPORTED;
  long long mtot = 0;
  for (int i = 0; i < n; ++i) {
    if (M[i] < 1 || !packed[i] || !scales[i] || !y[i]) return DK_ERR_INVALID_ARG;
    if (K > 0 && (!aligned16(packed[i]) || (reinterpret_cast<uintptr_t>(scales[i]) & 1u)))
      return DK_ERR_INVALID_ARG;
    if (reinterpret_cast<uintptr_t>(y[i]) & 1u) return DK_ERR_INVALID_ARG;
    mtot += M[i];
  }
  if (mtot > (1ll << 30)) return DK_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0) return DK_OK;
  if (K == 0) {
    for (int i = 0; i < n; ++i) {
      const cudaError_t e = cudaMemsetAsync(y[i], 0, (size_t)B * M[i] * sizeof(uint16_t), st);
      if (e != cudaSuccess) {
        set_cuda_error(e, "cudaMemsetAsync");
        return DK_ERR_CUDA;
      }
    }
    return DK_OK;
  }
  if (!x || !aligned16(x)) return DK_ERR_INVALID_ARG;
  const bool pdl = (c.flags & DK_FLAG_PDL) != 0;
  for (int b0 = 0; b0 < B; b0 += kMaxBatchPerPass) {
    GemvParams p;
    p.packed = reinterpret_cast<const uint32_t*>(packed[0]);
    p.scales = reinterpret_cast<const __half*>(scales[0]);
    p.x = reinterpret_cast<const __half*>(x) + (size_t)b0 * K;
    p.y = reinterpret_cast<__half*>(y[0]) + (size_t)b0 * M[0];
    p.M = (int)mtot;
    p.K = K;
    p.ldx = K;
    p.B = std::min(kMaxBatchPerPass, B - b0);
    p.ws = nullptr;
    p.counters = nullptr;
    SegList segs;
    std::memset(&segs, 0, sizeof(segs));
    segs.n = n;
    int tile0 = 0;
    for (int i = 0; i < n; ++i) {
      segs.s[i] = Segment{reinterpret_cast<const uint32_t*>(packed[i]),
                         reinterpret_cast<const __half*>(scales[i]),
                         reinterpret_cast<__half*>(y[i]) + (size_t)b0 * M[i], M[i], tile0};
      tile0 += (M[i] + 15) / 16;
    }
    const SegList* sl = n > 1 ? &segs : nullptr;  // one matrix: p already describes it
    s = c.reuse_weights ? launch_stream_nt<kStampReuse>(p, st, pdl, sl)
                        : launch_stream_nt<5>(p, st, pdl, sl);
    if (s != DK_OK) return s;
  }
  return DK_OK;
}

// ---------------------------------------------------------------------------
// Gate/up pair with the SiLU-mul epilogue: h = silu(x . Wg^T) * (x . Wu^T),
// the two GEMVs in one launch over (gate tile, up tile) pairs.
// ---------------------------------------------------------------------------
extern "C" dk_status dk_w4a16_gemv_silu_mul(const int32_t* packed_gate,
                                            const uint16_t* scales_gate,
                                            const int32_t* packed_up, const uint16_t* scales_up,
                                            const uint16_t* x, uint16_t* h, int M, int K, int B,
                                            const dk_gemv_config* cfg, void* stream) {
  stamp_begin_call();
  dk_gemv_config c;
  dk_gemv_config_init(&c);
  if (cfg) c = *cfg;
  dk_status s = validate_config(c);
  if (s != DK_OK) return s;
  if (c.flags & DK_FLAG_SHARD_WAIT) return DK_ERR_INVALID_ARG;
  if (M < 1 || K < 0 || B < 0 || K % DK_GROUP_SIZE != 0 || !packed_gate || !scales_gate ||
      !packed_up || !scales_up || !h)
    return DK_ERR_INVALID_ARG;
  if ((c.version != 5 && !c.reuse_weights) || (c.flags & DK_FLAG_F32_OUT)) return DK_ERR_UNSUPPORTED;
  if (K > 0 && (!aligned16(packed_gate) || !aligned16(packed_up) ||
                ((reinterpret_cast<uintptr_t>(scales_gate) | reinterpret_cast<uintptr_t>(scales_up)) & 1u)))
    return DK_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(h) & 1u) return DK_ERR_INVALID_ARG;
  if (2ll * M > (1ll << 30)) return DK_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0) return DK_OK;
  if (K == 0) {  // gate = up = 0, silu(0) * 0 = 0
    const cudaError_t e = cudaMemsetAsync(h, 0, (size_t)B * M * sizeof(uint16_t), st);
    if (e != cudaSuccess) {
      set_cuda_error(e, "cudaMemsetAsync");
      return DK_ERR_CUDA;
    }
    return DK_OK;
  }
  if (!x || !aligned16(x)) return DK_ERR_INVALID_ARG;
  const bool pdl = (c.flags & DK_FLAG_PDL) != 0;
  for (int b0 = 0; b0 < B; b0 += kMaxBatchPerPass) {
    GemvParams p;
    p.packed = reinterpret_cast<const uint32_t*>(packed_gate);
    p.scales = reinterpret_cast<const __half*>(scales_gate);
    p.x = reinterpret_cast<const __half*>(x) + (size_t)b0 * K;
    p.y = reinterpret_cast<__half*>(h) + (size_t)b0 * M;
    p.M = 2 * M;  // rows streamed
    p.K = K;
    p.ldx = K;
    p.B = std::min(kMaxBatchPerPass, B - b0);
    p.ws = nullptr;
    p.counters = nullptr;
    SegList segs;
    std::memset(&segs, 0, sizeof(segs));
    segs.n = 2;
    segs.paired = 1;
    segs.s[0] = Segment{reinterpret_cast<const uint32_t*>(packed_gate),
                        reinterpret_cast<const __half*>(scales_gate), p.y, M, 0};
    segs.s[1] = Segment{reinterpret_cast<const uint32_t*>(packed_up),
                        reinterpret_cast<const __half*>(scales_up), nullptr, M, 0};
    s = c.reuse_weights ? launch_stream_nt<kStampReuse>(p, st, pdl, &segs)
                        : launch_stream_nt<5>(p, st, pdl, &segs);
    if (s != DK_OK) return s;
  }
  return DK_OK;
}

// ---------------------------------------------------------------------------
// Sharded GEMV (row-parallel and K-parallel): the v5 pipeline with its
// epilogue storing into every rank's buffer and counting the rank in.
// ---------------------------------------------------------------------------
// CTAs of a sharded call: one per SM, or one per 16-row tile of `rows` if
// fewer; every rank derives it from the same numbers, so every rank has the
// same (a rank whose shard has fewer tiles leaves some CTAs without work;
// they still mark their arrival slots).
static int shard_grid(int rows) { return std::max(1, std::min(sm_count(-1), (rows + 15) / 16)); }

static dk_status shard_launch(GemvParams p, const dk_shard_group* g, const dk_gemv_config* cfg,
                              cudaStream_t st, bool fused_sum = false) {
  stamp_begin_call();
  dk_gemv_config c;
  dk_gemv_config_init(&c);
  if (cfg) c = *cfg;
  dk_status s = validate_config(c);
  if (s != DK_OK) return s;
  if (c.version != 5 || (c.flags & DK_FLAG_F32_OUT)) return DK_ERR_UNSUPPORTED;
  const bool kshard = p.out.mode == kOutKShard;
  const bool gather = p.out.mode == kOutRowGather;
  const bool await_all =
      kshard ? fused_sum : !gather && (c.flags & DK_FLAG_SHARD_WAIT) != 0;
  if (sm_count(-1) > DK_SHARD_SLOTS) return DK_ERR_UNSUPPORTED;
  if (!g || g->world < 1 || g->world > kMaxShards || g->rank < 0 || g->rank >= g->world ||
      !g->seq)
    return DK_ERR_INVALID_ARG;
  for (int i = 0; i < g->world; ++i)
    if (!g->bufs[i] || (!kshard && !gather && !g->slots[i]) ||
        (kshard && (reinterpret_cast<uintptr_t>(g->bufs[i]) & 7u)))
      return DK_ERR_INVALID_ARG;
  if (p.M <= 0 || p.K <= 0 || p.K % DK_GROUP_SIZE != 0 || p.B <= 0) return DK_ERR_INVALID_ARG;
  if (p.B > kMaxBatchPerPass) return DK_ERR_UNSUPPORTED;
  if (!p.packed || !p.scales || !p.x || !aligned16(p.packed) || !aligned16(p.x) ||
      (reinterpret_cast<uintptr_t>(p.scales) & 1u) || p.ldx < p.K || p.ldx % 8 != 0)
    return DK_ERR_INVALID_ARG;
  p.out.world = g->world;
  p.out.rank = g->rank;
  for (int i = 0; i < g->world; ++i) {
    p.out.dst[i] = g->bufs[i];
    p.out.slots[i] = g->slots[i];
  }
  p.out.seq = g->seq;
  p.out.await_all = await_all ? 1 : 0;
  p.ws = nullptr;
  p.counters = nullptr;
  if (!fused_sum) p.y = nullptr;
  const bool pdl = (c.flags & DK_FLAG_PDL) != 0;
  return c.reuse_weights ? launch_stream_nt<kStampReuse>(p, st, pdl)
                         : launch_stream_nt<5>(p, st, pdl);
}

extern "C" dk_status dk_w4a16_gemv_rowshard(const int32_t* packed, const uint16_t* scales,
                                            const uint16_t* x, int M_shard, int row0,
                                            int M_total, int K, int B,
                                            const dk_shard_group* group,
                                            const dk_gemv_config* cfg, void* stream) {
  stamp_begin_call();
  if (M_shard <= 0 || row0 < 0 || M_total < row0 + M_shard) return DK_ERR_INVALID_ARG;
  GemvParams p;
  p.packed = reinterpret_cast<const uint32_t*>(packed);
  p.scales = reinterpret_cast<const __half*>(scales);
  p.x = reinterpret_cast<const __half*>(x);
  p.M = M_shard;
  p.K = K;
  p.ldx = K;
  p.B = B;
  p.out.mode = kOutRowShard;
  p.out.ld = M_total;
  p.out.col0 = row0;
  if (group && group->world >= 1)  // the same on every rank: from the largest shard
    p.out.grid = shard_grid((M_total + group->world - 1) / group->world);
  return shard_launch(p, group, cfg, static_cast<cudaStream_t>(stream));
}

extern "C" dk_status dk_w4a16_gemv_kshard(const int32_t* packed, const uint16_t* scales,
                                          const uint16_t* x, int ldx, int M, int K_shard, int B,
                                          const dk_shard_group* group, const dk_gemv_config* cfg,
                                          void* stream) {
  GemvParams p;
  p.packed = reinterpret_cast<const uint32_t*>(packed);
  p.scales = reinterpret_cast<const __half*>(scales);
  p.x = reinterpret_cast<const __half*>(x);
  p.M = M;
  p.K = K_shard;
  p.ldx = ldx;
  p.B = B;
  p.out.mode = kOutKShard;
  p.out.ld = M;
  p.out.grid = shard_grid(M);
  return shard_launch(p, group, cfg, static_cast<cudaStream_t>(stream));
}

extern "C" dk_status dk_w4a16_gemv_rowshard_gather(const int32_t* packed, const uint16_t* scales,
                                                   const uint16_t* x, int M_shard, int row0,
                                                   int M_total, int K, int B,
                                                   const dk_shard_group* group, uint16_t* y,
                                                   const dk_gemv_config* cfg, void* stream) {
  stamp_begin_call();
  if (M_shard <= 0 || row0 < 0 || M_total < row0 + M_shard) return DK_ERR_INVALID_ARG;
  if (!y || (reinterpret_cast<uintptr_t>(y) & 1u)) return DK_ERR_INVALID_ARG;
  if (B > 8) return DK_ERR_UNSUPPORTED;  // one n-tile only (the row-shard call serves more)
  if (group)
    for (int i = 0; i < group->world && i < DK_MAX_SHARDS; ++i)
      if (reinterpret_cast<uintptr_t>(group->bufs[i]) & 7u) return DK_ERR_INVALID_ARG;
  GemvParams p;
  p.packed = reinterpret_cast<const uint32_t*>(packed);
  p.scales = reinterpret_cast<const __half*>(scales);
  p.x = reinterpret_cast<const __half*>(x);
  p.y = reinterpret_cast<__half*>(y);
  p.M = M_shard;
  p.K = K;
  p.ldx = K;
  p.B = B;
  p.out.mode = kOutRowGather;
  p.out.ld = M_total;
  p.out.col0 = row0;
  if (group && group->world >= 1)  // the same on every rank: from the largest shard
    p.out.grid = shard_grid((M_total + group->world - 1) / group->world);
  return shard_launch(p, group, cfg, static_cast<cudaStream_t>(stream), true);
}

extern "C" dk_status dk_w4a16_gemv_kshard_sum(const int32_t* packed, const uint16_t* scales,
                                              const uint16_t* x, int ldx, int M, int K_shard,
                                              int B, const dk_shard_group* group, uint16_t* y,
                                              const dk_gemv_config* cfg, void* stream) {
  stamp_begin_call();
  if (!y || (reinterpret_cast<uintptr_t>(y) & 1u)) return DK_ERR_INVALID_ARG;
  if (group && group->world >= 1 && (!group->seq)) return DK_ERR_INVALID_ARG;
  GemvParams p;
  p.packed = reinterpret_cast<const uint32_t*>(packed);
  p.scales = reinterpret_cast<const __half*>(scales);
  p.x = reinterpret_cast<const __half*>(x);
  p.y = reinterpret_cast<__half*>(y);
  p.M = M;
  p.K = K_shard;
  p.ldx = ldx;
  p.B = B;
  p.out.mode = kOutKShard;
  p.out.ld = M;
  p.out.grid = shard_grid(M);
  if (B <= 8) return shard_launch(p, group, cfg, static_cast<cudaStream_t>(stream), true);
  // 9..32 rows: the GEMV stores its partials, a separate kernel sums them (the same bits)
  const dk_status s = shard_launch(p, group, cfg, static_cast<cudaStream_t>(stream));
  if (s != DK_OK) return s;
  return dk_shard_reduce(group, M, B, y, 1, stream);
}

// ---------------------------------------------------------------------------
// Split-K without caller-provided memory.
//
// For callers that cannot allocate device memory at the point of the call --
// code running inside an allocator hook, a graph-capture region or a host
// runtime that owns every allocation itself -- the split-K path can use a
// fixed scratch buffer that lives in this library's own device image instead
// of a caller workspace.  Each device that loads the library holds it until
// the process exits.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_dk_noalloc_scratch[DK_NOALLOC_SCRATCH_BYTES];

static void* noalloc_scratch_ptr(dk_status* st) {
  // The symbol's device address, looked up once per device with that device
  // current (a host-side use of the symbol itself would not be a device
  // address).
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) {
    *st = DK_ERR_UNSUPPORTED;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_dk_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_cuda_error(e, "cudaGetSymbolAddress");
      *st = DK_ERR_CUDA;
      return nullptr;
    }
    ptrs[dev] = p;
  }
  *st = DK_OK;
  return ptrs[dev];
}

extern "C" dk_status dk_w4a16_gemv_splitk_noalloc(const int32_t* packed, const uint16_t* scales,
                                                  const uint16_t* x, uint16_t* y, int M, int K,
                                                  int B, int split_k, void* stream) {
  stamp_begin_call();
  dk_gemv_config c;
  dk_gemv_config_init(&c);
  c.version = 4;
  c.split_k = split_k;
  dk_status s = validate_config(c);
  if (s != DK_OK) return s;
  if (M < 0 || K < 0 || B < 0) return DK_ERR_INVALID_ARG;
  const size_t need = dk_w4a16_workspace_bytes(M, K, B, &c);
  if (need > (size_t)DK_NOALLOC_SCRATCH_BYTES) return DK_ERR_WORKSPACE;
  void* scratch = nullptr;
  if (need > 0) {
    scratch = noalloc_scratch_ptr(&s);
    if (s != DK_OK) return s;
  }
  // The split-K path clears the arrival counters at the start of every call,
  // so whatever the previous call left in the buffer does not matter.
  return dk_w4a16_gemv(packed, scales, x, y, M, K, B, &c, scratch,
                       need > 0 ? (size_t)DK_NOALLOC_SCRATCH_BYTES : 0, stream);
}

extern "C" int dk_last_kernel_stamp(int device) {
  int prev = -1;
  cudaGetDevice(&prev);
  if (device >= 0 && device != prev) cudaSetDevice(device);
  int h = -1;
  cudaDeviceSynchronize();
  if (!stamp_is_live(current_device()) ||
      cudaMemcpyFromSymbol(&h, g_dk_kernel_stamp, sizeof(int)) != cudaSuccess)
    h = -1;
  if (device >= 0 && device != prev) cudaSetDevice(prev);
  return h;
}

int* dk::device_error_address() {
  static std::mutex mu;
  static int* cache[64] = {nullptr};
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_dk_device_error);
  if (e != cudaSuccess) {
    set_cuda_error(e, "cudaGetSymbolAddress");
    return nullptr;
  }
  if (dev >= 0 && dev < 64) cache[dev] = static_cast<int*>(p);
  return static_cast<int*>(p);
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
