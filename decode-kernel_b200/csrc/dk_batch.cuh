// dk_batch.cuh -- the batch GEMV for 17..32 activation rows on large matrices,
// on the 5th-generation tensor cores (tcgen05).  Included by dk_gemv.cu after
// the v5 host helpers; serves version 5 and the weight-reuse path (see
// launch_batch for when it is taken).
//
// y[b, m] = sum_k x[b, k] * fp16(q[m, k] * scale[m, k / 128])
//
// Roles are swapped against a GEMM's usual "weights = A": the MMA's A operand
// is x (M = 128 lanes, batch row b in lane b, the lanes past B unused) and its
// B operand is the dequantized weight tile (N = up to 256 weight rows), so a
// CTA's whole row block is one N tile and the fp32 accumulator
// D[b][row] lives in tensor memory for the CTA's whole K loop.
//
// Per 128-k stage (one quantisation group), through rings as deep as shared
// memory allows (up to 8 stages of raw weights + x, up to 8 dequantized
// buffers):
//   producer warp   one TMA box of the tile's raw int4 rows (64 bytes each)
//                   and two 128-byte-swizzled boxes of x (32 rows x 64 k),
//                   all on one mbarrier;
//   8 dequant warps unpack each 8-weight word (LOP3 magic numbers, exact),
//                   restore natural k order (PRMT), fold in the group scale
//                   (HMUL2, one fp16 rounding) and store the fp16 tile in the
//                   K-major 128-byte-swizzle layout the MMA reads;
//   MMA warp        one elected thread issues 8 tcgen05.mma (k = 16 each)
//                   and commits them to the barriers that free the buffers;
//   the producer warp, once its copies are issued, reads D back (tcgen05.ld)
//   after the last commit and writes y.
// Numerics: the weight is rounded once to fp16 (q * scale), products and
// sums are fp32 on the tensor core; the result is within the 1e-2 tolerance
// but is not bit-identical to the B <= 8 kernels, whose canonical order
// scales each group's fp32 dot product instead.
namespace vb {
constexpr int kChunkK = 128;                        // one group per stage
constexpr int kRawRowBytes = kChunkK / 2;           // 64 bytes of int4 per row
constexpr int kAtomK = 64;                          // fp16 k per 128-byte swizzled row
constexpr int kAtoms = kChunkK / kAtomK;            // 2
constexpr int kXRows = 32;                          // batch rows staged per pass
constexpr int kXAtomBytes = kXRows * 128;           // 4 KB
constexpr int kXStageBytes = kAtoms * kXAtomBytes;  // 8 KB
constexpr int kMmaM = 128;
constexpr int kMaxN = 256;
constexpr int kMaxStages = 8;  // raw weight + x ring
constexpr int kMaxBBufs = 8;   // dequantized weight ring
constexpr int kBudget = 208 * 1024;
constexpr int kDqWarps = 8;
constexpr int kProducerWarp = kDqWarps;  // also the epilogue warp: lanes 0-31 of D
constexpr int kMmaWarp = kDqWarps + 1;
constexpr int kThreads = (kDqWarps + 2) * 32;
// Tensor-memory columns for an N-wide fp32 accumulator: a power of two >= 32.
__host__ __device__ constexpr uint32_t tmem_cols(int ntile) {
  return ntile <= 32 ? 32u : ntile <= 64 ? 64u : ntile <= 128 ? 128u : 256u;
}
// Independent accumulators the MMAs rotate over (k step i goes to i % nacc),
// so consecutive MMAs do not wait on each other's result; they are added in
// order 0..nacc-1 when read back.  As many as fit in 256 columns, up to 4.
__host__ __device__ constexpr int num_acc(int ntile) {
  return tmem_cols(ntile) <= 64 ? 4 : tmem_cols(ntile) == 128 ? 2 : 1;
}
// The MMA reads 128 A rows per atom, 16 KB from the atom's start; only the
// first 32 are x, the rest land on the buffers that follow the x ring (their
// lanes' results are never read).  The weight buffers are at least this large.
constexpr int kATail = kMmaM * 128 - kXAtomBytes;

// nst stages of raw weights + x, nbb buffers of dequantized weights, and the
// CTA's whole block of scales (ntile rows x all groups), staged once.
constexpr int kMaxScaleBytes = 64 * 1024;
__host__ __device__ inline int scale_bytes(int ntile, int groups) {
  return (ntile * groups * 2 + 127) / 128 * 128;
}
struct Layout {
  int x_off, b_off, raw_off, sc_off, bar_off, total;
};
__host__ __device__ inline Layout layout(int ntile, int nst, int nbb, int groups) {
  Layout L;
  int off = 0;
  L.x_off = off;
  off += nst * kXStageBytes;
  L.b_off = off;
  off += max(nbb * ntile * kChunkK * 2, kATail + 1024);
  L.raw_off = off;
  off += (nst * ntile * kRawRowBytes + 127) / 128 * 128;
  L.sc_off = off;
  off += scale_bytes(ntile, groups);
  L.bar_off = off;
  off += (3 * kMaxStages + 2 * kMaxBBufs + 3) * 8 + 16;  // full, raw_free, x_free, bfull, bfree, acc, mma_done, tmem slot + flag
  L.total = off;
  return L;
}
// Deepest rings that fit: the chain "copy -> dequantize -> MMA -> commit"
// is latency-bound per stage, so depth is what keeps the tensor cores fed.
__host__ inline void rings(int ntile, int nk, int* nst, int* nbb) {
  const int per_stage = ntile * kRawRowBytes + kXStageBytes, bbuf = ntile * kChunkK * 2;
  const int budget = kBudget - scale_bytes(ntile, nk);  // one group per stage: groups == nk
  int r = kMaxStages;
  while (r > 2 && r * per_stage + 2 * bbuf > budget) --r;
  int b = std::min(kMaxBBufs, std::max(2, (budget - r * per_stage) / bbuf));
  *nst = std::max(1, std::min(r, nk));
  *nbb = std::max(1, std::min(b, nk));
}
}  // namespace vb

template <int STAMP>
__global__ void __launch_bounds__(vb::kThreads, 1)
    k_batch(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
            GemvParams p, int ntile, int nst, int nbb) {
  using namespace vb;
  extern __shared__ __align__(1024) uint8_t smem[];
  const Layout L = layout(ntile, nst, nbb, p.K / kGroup);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);  // [nst] copies landed
  uint64_t* raw_free = full + kMaxStages;    // [nst] dequant warps read the raw tile
  uint64_t* x_free = raw_free + kMaxStages;  // [nst] MMAs that read the x tile completed
  uint64_t* bfull = x_free + kMaxStages;     // [nbb] dequantized tile stored
  uint64_t* bfree = bfull + kMaxBBufs;       // [nbb] MMAs that read it completed
  uint64_t* acc_full = bfree + kMaxBBufs;    // every MMA of the tile completed
  uint64_t* mma_done = acc_full + 1;      // every MMA issued completed (teardown)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const uint32_t xbase = smem_u32(smem + L.x_off), bbase = smem_u32(smem + L.b_off);
  const uint32_t rawbase = smem_u32(smem + L.raw_off);
  __half* scs = reinterpret_cast<__half*>(smem + L.sc_off);  // [ntile][groups]
  write_stamp(STAMP);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = (int)(((long long)blockIdx.x * p.M) / gridDim.x);
  const int r1 = (int)(((long long)(blockIdx.x + 1) * p.M) / gridDim.x);
  const int groups = p.K / kGroup;
  const int nk = p.K / kChunkK;
  const uint32_t raw_stage = (uint32_t)ntile * kRawRowBytes;
  const uint32_t b_buf = (uint32_t)ntile * kChunkK * 2;  // two atoms of ntile rows x 128 B
  const uint32_t b_atom = (uint32_t)ntile * 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&raw_free[s], kDqWarps);
      mbar_init(&x_free[s], 1);
    }
    for (int b = 0; b < nbb; ++b) {
      mbar_init(&bfull[b], kDqWarps);
      mbar_init(&bfree[b], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&wmap);
    tma_prefetch_desc(&xmap);
  }
  const int nacc = num_acc(ntile);
  const uint32_t acc_cols = tmem_cols(ntile), alloc_cols = acc_cols * (uint32_t)nacc;
  if (warp == kMmaWarp) tmem_alloc(smem_u32(tmem_slot), alloc_cols);
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == kProducerWarp) {
    // ---------------- copies, then the epilogue ----------------
    int issued = 0;
    if (lane == 0) {
      const uint64_t wpol = policy_evict_first(), xpol = policy_evict_last();
      const uint32_t bytes = raw_stage + kXStageBytes;
      const int pre = min(nst, nk);
      // Weights never come from the predecessor grid: stream them first.
      for (int s = 0; s < pre; ++s) {
        mbar_arrive_expect_tx(&full[s], bytes);
        tma_load_2d(rawbase + s * raw_stage, &wmap, s * kRawRowBytes, r0, &full[s], wpol);
      }
      pdl_wait();  // x and y belong to the predecessor until here
      for (int s = 0; s < pre; ++s)
        for (int a = 0; a < kAtoms; ++a)
          tma_load_2d(xbase + s * kXStageBytes + a * kXAtomBytes, &xmap,
                      s * kChunkK + a * kAtomK, 0, &full[s], xpol);
      issued = pre;
      for (int s = pre; s < nk; ++s) {
        const int slot = s % nst, ph = ((s / nst) - 1) & 1;
        if (!mbar_wait_spin_bounded(&raw_free[slot], ph, abort_flag)) break;
        if (!mbar_wait_spin_bounded(&x_free[slot], ph, abort_flag)) break;
        mbar_arrive_expect_tx(&full[slot], bytes);
        tma_load_2d(rawbase + slot * raw_stage, &wmap, s * kRawRowBytes, r0, &full[slot], wpol);
        for (int a = 0; a < kAtoms; ++a)
          tma_load_2d(xbase + slot * kXStageBytes + a * kXAtomBytes, &xmap,
                      s * kChunkK + a * kAtomK, 0, &full[slot], xpol);
        issued = s + 1;
      }
    }
    issued = __shfl_sync(0xffffffffu, issued, 0);
    __syncwarp();
    // Epilogue: lane b holds batch row b's accumulators, column j = row r0 + j.
    if (mbar_wait_spin_bounded(acc_full, 0, abort_flag)) {
      tcgen05_fence_after();
      const int rows = r1 - r0;
      for (int c0 = 0; c0 < ntile; c0 += 16) {
        float acc[16];
        for (int a = 0; a < nacc; ++a) {
          uint32_t v[16];
          tmem_ld16(tmem + (uint32_t)a * acc_cols + (uint32_t)c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            acc[j] = a == 0 ? __uint_as_float(v[j]) : __fadd_rn(acc[j], __uint_as_float(v[j]));
        }
        if (lane < p.B) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < rows) store_y<false>(p, lane, r0 + c0 + j, acc[j]);
        }
      }
      tcgen05_fence_before();
      signal_shards(p, lane);
    }
    if (*abort_flag && lane == 0) {
      volatile int no_abort = 0;
      for (int s = max(0, issued - nst); s < issued; ++s)
        mbar_wait_spin_bounded(&full[s % nst], (s / nst) & 1, &no_abort);
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issue (one thread) ----------------
    if (lane == 0) {
      // kind::f16 instruction descriptor: fp32 accumulator, A = B = fp16,
      // both K-major, N = ntile, M = 128.
      const uint32_t idesc = (1u << 4) | ((uint32_t)(ntile >> 3) << 17) |
                             ((uint32_t)(kMmaM >> 4) << 24);
      for (int s = 0; s < nk; ++s) {
        const int slot = s % nst, b = s % nbb;
        if (!mbar_wait_spin_bounded(&bfull[b], (s / nbb) & 1, abort_flag)) break;
        if (!mbar_wait_spin_bounded(&full[slot], (s / nst) & 1, abort_flag)) break;
        tcgen05_fence_after();
        const uint32_t xa = xbase + slot * kXStageBytes, wb = bbase + b * b_buf;
#pragma unroll
        for (int a = 0; a < kAtoms; ++a)
#pragma unroll
          for (int k = 0; k < kAtomK / 16; ++k) {
            const int i = s * (kAtoms * kAtomK / 16) + a * (kAtomK / 16) + k;  // k step
            umma_f16(tmem + (uint32_t)(i % nacc) * acc_cols,
                     umma_desc_k_sw128(xa + a * kXAtomBytes + k * 32),
                     umma_desc_k_sw128(wb + a * b_atom + k * 32), idesc, i >= nacc);
          }
        umma_commit(&x_free[slot]);
        umma_commit(&bfree[b]);
        if (s == nk - 1) umma_commit(acc_full);
      }
      // Every MMA issued has completed before tensor memory is released.
      umma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait_spin_bounded(mma_done, 0, &no_abort);
    }
    __syncwarp();
  } else {
    // ---------------- dequantisation (8 warps) ----------------
    const int t = threadIdx.x;  // 0 .. 255
    const int words = ntile * (kChunkK / 8);
    {
      // The tile's scales, once (never the predecessor's output: no PDL
      // wait); consecutive threads take consecutive groups of a row.
      const int n_sc = ntile * groups;
      for (int i = t; i < n_sc; i += kDqWarps * 32) {
        const int n = i / groups, g = i - n * groups;
        scs[i] = __ldg(p.scales + (size_t)min(r0 + n, p.M - 1) * groups + g);
      }
      named_barrier(1, kDqWarps * 32);
    }
    for (int s = 0; s < nk; ++s) {
      const int slot = s % nst, b = s % nbb;
      if (!mbar_wait_spin_bounded(&full[slot], (s / nst) & 1, abort_flag)) break;
      if (s >= nbb && !mbar_wait_spin_bounded(&bfree[b], ((s / nbb) - 1) & 1, abort_flag)) break;
      const uint32_t raw = rawbase + slot * raw_stage, dst = bbase + b * b_buf;
      // Four words of one row per trip (one 16-byte load, one scale, four
      // independent unpack chains): quad u = 4n + v holds words 4v .. 4v + 3
      // of tile row n, all in swizzle atom v / 2.
      for (int u = t; u < words / 4; u += kDqWarps * 32) {
        const int n = u >> 2, w0 = (u & 3) << 2;  // tile row n, words w0 .. w0 + 3
        const uint4 wq = lds128(raw + n * kRawRowBytes + w0 * 4);
        const uint32_t wv[4] = {wq.x, wq.y, wq.z, wq.w};
        const __half sc = scs[n * groups + s];
        const __half2 s2 = __halves2half2(sc, sc);
        const uint32_t row = dst + (w0 >> 3) * b_atom + (n >> 3) * 1024 + (n & 7) * 128;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint32_t h[4];
          unpack_q8(wv[e], h);  // (q0,q4), (q1,q5), (q2,q6), (q3,q7)
          uint32_t o[4] = {prmt(h[0], h[1], 0x5410u), prmt(h[2], h[3], 0x5410u),
                           prmt(h[0], h[1], 0x7632u), prmt(h[2], h[3], 0x7632u)};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const __half2 v = __hmul2(*reinterpret_cast<const __half2*>(&o[i]), s2);
            o[i] = *reinterpret_cast<const uint32_t*>(&v);
          }
          const int j = (w0 & 7) + e;  // 16-byte chunk of the 128-byte swizzled row
          sts128(row + ((j ^ (n & 7)) << 4), o);
        }
      }
      fence_async_shared();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&raw_free[slot]);
        mbar_arrive(&bfull[b]);
      }
    }
  }

  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, alloc_cols);
}

// x as a 2-D tensor map {K, B} of fp16 with 64 x 32 boxes and the 128-byte
// swizzle (rows past B read as zero).  Cached per (pointer, K, B).
bool x_tensor_map(const void* x, int K, int B, CUtensorMap* out) {
  struct Entry {
    const void* ptr;
    int K, B;
    unsigned long long stamp;
    CUtensorMap map;
  };
  static std::mutex mu;
  static Entry cache[64];
  static unsigned long long clock = 0;
  std::lock_guard<std::mutex> lk(mu);
  Entry* victim = &cache[0];
  for (Entry& e : cache) {
    if (e.stamp && e.ptr == x && e.K == K && e.B == B) {
      e.stamp = ++clock;
      *out = e.map;
      return true;
    }
    if (e.stamp < victim->stamp) victim = &e;
  }
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)B};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)vb::kAtomK, (cuuint32_t)vb::kXRows};
  cuuint32_t elem[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(x), dims, strides, box, elem,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  *victim = Entry{x, K, B, ++clock, map};
  *out = map;
  return true;
}

// The weights as a 2-D tensor map {K/2 bytes, M rows} with 64-byte x ntile
// boxes, no swizzle (the dequant warps read whole words).  Cached per
// (pointer, M, K, ntile).
bool raw_tensor_map(const void* packed, int M, int K, int ntile, CUtensorMap* out) {
  struct Entry {
    const void* ptr;
    int M, K, ntile;
    unsigned long long stamp;
    CUtensorMap map;
  };
  static std::mutex mu;
  static Entry cache[64];
  static unsigned long long clock = 0;
  std::lock_guard<std::mutex> lk(mu);
  Entry* victim = &cache[0];
  for (Entry& e : cache) {
    if (e.stamp && e.ptr == packed && e.M == M && e.K == K && e.ntile == ntile) {
      e.stamp = ++clock;
      *out = e.map;
      return true;
    }
    if (e.stamp < victim->stamp) victim = &e;
  }
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)K / 2, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)K / 2};
  cuuint32_t box[2] = {(cuuint32_t)vb::kRawRowBytes, (cuuint32_t)ntile};
  cuuint32_t elem[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(packed), dims, strides, box,
          elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  *victim = Entry{packed, M, K, ntile, ++clock, map};
  *out = map;
  return true;
}

// Taken for B in 17..32 on matrices of at least kMinRows rows, plain outputs
// (fp16 or fp32), K a multiple of 128; DK_ERR_UNSUPPORTED otherwise and the
// caller takes the mma.sync streaming kernel.  Measured on B200: every MMA
// here reads its 128-row A operand (x, mostly padding) from shared memory, so
// a 128-k stage costs ~1200-1900 cycles however few weight rows the CTA owns;
// that beats the streaming kernel's 4 n-tiles only when the CTA's share of W
// is large (28672x8192, B=32: 112 vs 247 us) and loses on small matrices
// (4096x4096, B=32: 34 vs 25 us).
constexpr int kMinRows = 16384;
template <int STAMP>
dk_status launch_batch(GemvParams p, cudaStream_t st, bool pdl) {
  using namespace vb;
  if (p.B <= 16 || p.B > kXRows || p.M < kMinRows || p.out.mode > kOutFloat ||
      p.ldx != p.K || p.K % kChunkK != 0)
    return DK_ERR_UNSUPPORTED;
  const int sms = sm_count(-1);
  const int grid = std::max(std::min(sms, (p.M + 15) / 16), (p.M + kMaxN - 1) / kMaxN);
  const int rows = (p.M + grid - 1) / grid;
  const int ntile = std::min(kMaxN, (rows + 15) / 16 * 16);
  if (scale_bytes(ntile, p.K / kGroup) > kMaxScaleBytes) return DK_ERR_UNSUPPORTED;
  int nst = 0, nbb = 0;
  rings(ntile, p.K / kChunkK, &nst, &nbb);
  const size_t smem = layout(ntile, nst, nbb, p.K / kGroup).total;
  if (smem > (size_t)v5::kSmemCap) return DK_ERR_UNSUPPORTED;
  CUtensorMap wmap, xmap;
  if (!raw_tensor_map(p.packed, p.M, p.K, ntile, &wmap) || !x_tensor_map(p.x, p.K, p.B, &xmap))
    return DK_ERR_UNSUPPORTED;
  static std::atomic<unsigned long long> smem_done{0};
  dk_status s = ensure_smem(k_batch<STAMP>, v5::kSmemCap, smem_done);
  if (s != DK_OK) return s;
  return launch("k_batch", k_batch<STAMP>, dim3(grid), dim3(kThreads), smem, st, pdl, wmap, xmap,
                p, ntile, nst, nbb);
}
