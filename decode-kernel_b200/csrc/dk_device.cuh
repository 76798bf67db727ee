// dk_device.cuh -- device-side building blocks shared by the W4A16 kernels.
//
// Everything here is sm_100a device code written directly in PTX where the
// instruction matters: the LOP3 nibble-to-fp16 unpack, the m16n8k16 HMMA used
// as an fp32-accumulating dot-product unit, mbarrier waits with an iteration
// and wall-clock bound, TMA copies (tensor-map boxes and 1-D bulk copies),
// cp.async completion on mbarriers and the programmatic-dependent-launch
// controls.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dk {

constexpr int kGroup = 128;      // weights per fp16 scale (gemv_w4a16.h:9)
constexpr int kNibbles = 8;      // nibbles per packed word (gemv_w4a16.h:10)
constexpr int kWordsPerGroup = kGroup / kNibbles;  // 16 words = 64 bytes

// Device error word, one per device (a module global is per context).
// Written with the first error a kernel detects; read by dk_device_error().
enum DeviceError : int {
  kDevOk = 0,
  kDevWaitTimeout = 1,  // an mbarrier / flag wait exceeded its bound
};

#ifdef DK_DEVICE_GLOBALS
// Defined in exactly one translation unit (dk_gemv.cu), which is the only one
// whose kernels record stamps or bounded-wait errors.
__device__ int g_dk_device_error = 0;

// Dispatch stamp: which GEMV kernel ran last on this device
// (gemv_w4a16.cu:18-25 keeps the same contract).
__device__ int g_dk_kernel_stamp = -1;

__device__ __forceinline__ void write_stamp(int v) {
  if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 0) {
    g_dk_kernel_stamp = v;
  }
}
#endif

// ---------------------------------------------------------------------------
// Nibble unpack.  A packed word holds q0..q7 (signed 4-bit, two's complement,
// q_n at bits 4n).  One LOP3 per half2 builds an fp16 whose mantissa is the
// nibble with its sign bit flipped, under exponent 2^10:
//   lut 0x6A computes (b & (a ^ c)) | (~b & c): bits selected by the mask b
//   copy a, except where c is also set (bit 3 of the nibble), which flips it;
//   bits only in c (the 0x6400 exponent pattern) are forced to 1.
// Low nibbles (bits 0-3 / 16-19) give 1024 + (q + 8); one HSUB2 by 1032 gives
// q exactly.  High nibbles of a byte (bits 4-7 / 20-23) give 1024 + 16(q + 8);
// one HFMA2 by (1/16, -72) gives q exactly.  A shift by 8 exposes the other
// two nibble pairs.  Result, as four half2 (low half first):
//   h[0] = (q0, q4), h[1] = (q1, q5), h[2] = (q2, q6), h[3] = (q3, q7).
// 9 instructions per 8 weights; every value is exact.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lop3_6a(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ void unpack_q8(uint32_t w, uint32_t (&h)[4]) {
  constexpr uint32_t kLoMask = 0x000F000Fu, kLoMagic = 0x64086408u;  // 1032
  constexpr uint32_t kHiMask = 0x00F000F0u, kHiMagic = 0x64806480u;
  constexpr uint32_t kSixteenth = 0x2C002C00u;  // (1/16, 1/16)
  constexpr uint32_t kMinus72 = 0xD480D480u;    // (-72, -72)
  const uint32_t w8 = w >> 8;
  h[0] = hsub2_u32(lop3_6a(w, kLoMask, kLoMagic), kLoMagic);
  h[1] = hfma2_u32(lop3_6a(w, kHiMask, kHiMagic), kSixteenth, kMinus72);
  h[2] = hsub2_u32(lop3_6a(w8, kLoMask, kLoMagic), kLoMagic);
  h[3] = hfma2_u32(lop3_6a(w8, kHiMask, kHiMagic), kSixteenth, kMinus72);
}

// Byte permute: d = bytes {a, b}[sel].
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// x0..x7 (four half2 registers r0..r3 = (x0,x1),(x2,x3),(x4,x5),(x6,x7)) into
// the pair order that matches unpack_q8: (x0,x4),(x1,x5),(x2,x6),(x3,x7).
__device__ __forceinline__ void pair_x8(const uint4& r, uint32_t (&p)[4]) {
  p[0] = prmt(r.x, r.z, 0x5410);
  p[1] = prmt(r.x, r.z, 0x7632);
  p[2] = prmt(r.y, r.w, 0x5410);
  p[3] = prmt(r.y, r.w, 0x7632);
}

// ---------------------------------------------------------------------------
// HMMA m16n8k16, fp16 inputs, fp32 accumulate.  Used as the dot-product unit:
// A = 16 weight rows, B = up to 8 batch columns of x.
// Fragment ownership (lane = 4g + c):
//   A: a0a1 (row g, k 2c..2c+1) a2a3 (row g+8, k 2c..) a4a5 (row g, k 2c+8..)
//      a6a7 (row g+8, k 2c+8..)
//   B: b0b1 (k 2c..2c+1, col g) b2b3 (k 2c+8.., col g)
//   D: d0d1 (row g, cols 2c, 2c+1) d2d3 (row g+8, cols 2c, 2c+1)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                         uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// Global loads.
// ---------------------------------------------------------------------------
// Streamed-once data (packed weights): non-coherent path, no L1 allocation.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Data another grid may have just written (x after a PDL wait): L2 only.
__device__ __forceinline__ uint4 ldcg128(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}

// Re-read data (x, scales): default caching so other warps hit L1.
__device__ __forceinline__ uint4 ldg_keep(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ float ldg_half(const __half* p) {
  return __half2float(__ldg(p));
}

// ---------------------------------------------------------------------------
// Shared memory, mbarriers, bulk copies.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(addr));
  return r;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Make barrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps (up to `ns`) instead of spinning through issue slots.
// Non-blocking phase test.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Warp-uniform non-blocking test: lane 0 tests (acquire), the warp follows
// it past a __syncwarp so every lane is ordered after the phase.
__device__ __forceinline__ bool warp_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_test_wait(bar, parity) ? 1u : 0u;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  __syncwarp();
  return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every wait in this library is bounded: 2 s of wall clock.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Sharded calls: a release store of `epoch` into another GPU's (or this
// GPU's) arrival slot, and the warp-wide wait until slots[r * stride + b] >=
// epoch (wrap-safe) for every r < world, b < grid.  The wait polls with
// relaxed system-scope loads (independent, so they overlap) and, once every
// slot is marked, each lane issues an acquire fence, which with the release
// stores orders everything the marking CTAs stored before what follows.  On
// timeout it records kDevWaitTimeout in *err and returns false.  Call the
// wait with all 32 lanes.
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Low-latency exchange words: a value and the call's sequence number in one
// naturally aligned 64-bit word, stored and loaded as single 64-bit accesses
// (single-copy atomic, also across NVLink), so a reader that sees the number
// sees the value with it -- no fence between data and flag.
__device__ __forceinline__ void st_ll_sys(unsigned long long* p, float v, unsigned tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_ll_sys(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

__device__ inline bool wait_slots(const unsigned* slots, int stride, int world, int grid,
                                  unsigned epoch, int* err) {
  const int lane = threadIdx.x & 31;
  const int n = world * grid;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    bool mine = true;
    for (int i = lane; i < n; i += 32) {
      const int r = i / grid, b = i - r * grid;
      mine &= (int)(ld_relaxed_sys_u32(slots + r * stride + b) - epoch) >= 0;
    }
    if (__all_sync(0xffffffffu, mine)) {
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      return true;
    }
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      if (lane == 0) atomicExch(err, 1);
      return false;
    }
    __nanosleep(32);
  }
}

#ifdef DK_DEVICE_GLOBALS
// A wait that runs out records kDevWaitTimeout in g_dk_device_error, raises
// the CTA's abort flag (so every other wait in the CTA returns at once) and
// returns false.

// Same bound, polling with the non-suspending test: for barriers completed by
// tensor-core commits, where the waiter should resume the moment they land.
__device__ __forceinline__ bool mbar_wait_spin_bounded(uint64_t* bar, uint32_t parity,
                                                       volatile int* abort_flag) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (int i = 0;; ++i) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((i & 63) == 63) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicExch(&g_dk_device_error, kDevWaitTimeout);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Same bound, polling with the non-suspending test and a short sleep between
// tests: for a wait whose end is latency-critical (a suspended warp resumes
// late) but that should still leave most issue slots to the other warps of
// its sub-partition.
__device__ __forceinline__ bool mbar_wait_poll_bounded(uint64_t* bar, uint32_t parity,
                                                       volatile int* abort_flag) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (int i = 0;; ++i) {
    __nanosleep(32);
    if (mbar_test_wait(bar, parity)) return true;
    if ((i & 63) == 63) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicExch(&g_dk_device_error, kDevWaitTimeout);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_sleep(bar, parity, 200000u)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      atomicExch(&g_dk_device_error, kDevWaitTimeout);
      *abort_flag = 1;
      return false;
    }
  }
}

#endif  // DK_DEVICE_GLOBALS

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` of
// transaction count on `bar`.  dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst_smem, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst_smem),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Tensor-map TMA load of a 3-D box into this CTA's shared memory, completing
// the box's bytes of transaction count on `bar`.  c0 is the innermost
// coordinate (bytes inside a 128-byte strip; always 0 here, so 16-byte
// aligned).  Box parts outside the tensor are zero-filled.
__device__ __forceinline__ void tma_load_3d(uint32_t dst_smem, const void* tmap, int c0, int c1,
                                            int c2, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst_smem),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst_smem, const void* tmap, int c0, int c1,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst_smem),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------------------
// 5th-generation tensor cores (tcgen05): tensor-memory allocation, the
// single-thread MMA issue, its completion signal and the accumulator read.
// ---------------------------------------------------------------------------
// Allocate `ncols` (a power of two >= 32) tensor-memory columns; the address
// is written to shared memory at `dst`.  Whole warp.
__device__ __forceinline__ void tmem_alloc(uint32_t dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, kind::f16, one thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}
// Arrive on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tcgen05_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tcgen05_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes, made visible to the async proxy (the
// tensor cores and TMA) before a barrier hands the buffer over.
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 16 consecutive fp32 columns of this warp's 32 lanes (lane = thread).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Shared-memory matrix descriptor of a K-major operand in the 128-byte
// swizzle layout: rows of 128 bytes (64 fp16 of K), 8-row atoms 1024 bytes
// apart; `addr` is where the MMA's 16-k slice starts.
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);  // start address (16-byte units)
  d |= (uint64_t)1 << 16;                  // leading byte offset (unused for this layout)
  d |= (uint64_t)(1024 >> 4) << 32;        // stride byte offset: next 8-row atom
  d |= (uint64_t)1 << 46;                  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                  // layout: 128-byte swizzle
  return d;
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

__device__ __forceinline__ void sts128(uint32_t addr, const uint32_t (&v)[4]) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
}

__device__ __forceinline__ float lds_half(uint32_t addr) {
  unsigned short h;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(addr));
  return __half2float(__ushort_as_half(h));
}

// 4-byte Ampere-style async copy global -> shared (through L1).
__device__ __forceinline__ void cp_async4(uint32_t dst_smem, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst_smem), "l"(src) : "memory");
}

// Arrives on `bar` once every cp.async this thread issued so far has landed;
// counts toward the barrier's expected arrivals (no pending-count increment).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// L2 policy for data every CTA re-reads (the activations).
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// L2 policy for data read exactly once per call (the packed weights).
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Named barrier over a subset of warps (id 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialisation attribute may start before its predecessor finishes;
// it must call pdl_wait() before touching memory the predecessor writes or
// reads.  Without the attribute both are no-ops.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace dk
