/*
 * dk_w4a16.h -- C ABI of the B200 (sm_100a) W4A16 decode-GEMV library.
 *
 * This is the drop-in boundary for RohanDisa/decode-kernel's GEMV path.  The
 * reference exposes it as C++ functions in namespace decode_kernel
 * (include/decode_kernel/gemv_w4a16.h) bound to Python by a torch extension
 * (csrc/bindings.cpp).  Here the same operations are plain extern "C"
 * functions over raw pointers and sizes -- no torch or C++ types -- so any
 * FFI (ctypes, cffi, cgo, JNI) can bind them; this repository's torch
 * extension `decode_kernel._cuda` is one such caller.
 *
 * Data format (gemv_w4a16.h:29-33, python/decode_kernel/quantize.py:1-15):
 *   packed  int32   [M, K/8]   8 signed 4-bit values per word, value k%8 at
 *                               bits 4*(k%8) (low nibble first), two's
 *                               complement.
 *   scales  fp16    [M, K/128] one scale per 128 consecutive k of a row.
 *   x       fp16    [B, K]
 *   y       fp16    [B, M]     y[b,m] = sum_k x[b,k] * q[m,k] * scale[m,k/128]
 * All matrices are row-major and contiguous.  fp16 values are passed as their
 * IEEE binary16 bit patterns (uint16_t).  K must be a multiple of 128.
 * `packed` and `x` must be 16-byte aligned (any fresh cudaMalloc/torch
 * allocation is).
 *
 * Streams are cudaStream_t passed as void* (NULL = legacy default stream).
 * Every call is asynchronous on that stream, allocates nothing, and returns a
 * status; device-side faults surface on the stream as usual.
 */
#ifndef DK_W4A16_H_
#define DK_W4A16_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DK_API __attribute__((visibility("default")))
#else
#define DK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* gemv_w4a16.h:9-11 (kGroupSize, kNibblesPerWord, kWeightsPerInt4). */
#define DK_GROUP_SIZE 128
#define DK_NIBBLES_PER_WORD 8
#define DK_WEIGHTS_PER_INT4 32

/* Status of every call.  The reference prints launch errors and carries on
 * (gemv_w4a16.cu:9-16); this ABI reports them. */
typedef enum dk_status {
  DK_OK = 0,
  DK_ERR_INVALID_ARG = 1,  /* shape, range or alignment rejected */
  DK_ERR_UNSUPPORTED = 2,  /* valid request this build cannot serve */
  DK_ERR_LAUNCH = 3,       /* cudaLaunch* failed; see dk_last_cuda_error() */
  DK_ERR_TIMEOUT = 4,      /* a bounded device wait ran out */
  DK_ERR_CUDA = 5,         /* another CUDA runtime call failed */
  DK_ERR_WORKSPACE = 6     /* workspace missing or smaller than required */
} dk_status;

/* gemv_w4a16.h:13-20 KernelVersion: the six entries of the reference's kernel
 * family, each served by its own sm_100a kernel here. */
typedef enum dk_kernel_version {
  DK_V0_ROW_SCALAR = 0,   /* one thread per row */
  DK_V1_WARP_ROW = 1,     /* one warp (or block) per row, CUDA cores */
  DK_V2_TILE_DIRECT = 2,  /* 16-row tensor-core tiles, 128-bit register loads */
  DK_V3_TILE_SCALES = 3,  /* v2 with the tile's scales staged in shared memory */
  DK_V4_SPLIT_K = 4,      /* v2 split along K across CTAs, fp32 workspace */
  DK_V5_STREAM = 5        /* persistent bulk-copy pipeline (default, fastest) */
} dk_kernel_version;

/* Launch flags (no counterpart in the reference). */
#define DK_FLAG_PDL 0x1u /* launch with programmatic stream serialisation: the
                          * kernel may start while the previous kernel on the
                          * stream drains and streams its WEIGHTS before waiting
                          * for it; x and y are touched only after the wait.
                          * Only valid when the previous kernel on the stream
                          * does not write `packed` or `scales`. */

#define DK_FLAG_F32_OUT 0x2u /* version 5 (and the reuse path) only: y is fp32
                              * [B, M] -- pass the float pointer as `y` -- with
                              * no rounding to fp16.  Other versions return
                              * DK_ERR_UNSUPPORTED. */

#define DK_FLAG_SHARD_WAIT 0x4u /* sharded calls only: the call completes on the
                                 * stream only once every rank's part has
                                 * arrived here (CTA 0 waits, bounded, and
                                 * advances group->seq), so no dk_shard_wait
                                 * is needed.  Only for ranks on
                                 * different GPUs running concurrently: ranks
                                 * that share one GPU and one stream must use
                                 * dk_shard_wait instead. */

/* gemv_w4a16.h:22-27 GemvLaunchConfig, same fields and defaults, plus flags. */
typedef struct dk_gemv_config {
  int version;       /* 0..5, default 5 */
  int split_k;       /* 1..32, default 4; version 4 only */
  int reuse_weights; /* default 0; non-zero selects the batch weight-reuse path */
  int warps_per_row; /* 1..8, default 1; >1 only with version 1, no reuse */
  unsigned flags;    /* DK_FLAG_* */
} dk_gemv_config;

/* Fills the reference defaults (version 5, split_k 4, no reuse, 1 warp/row). */
DK_API void dk_gemv_config_init(dk_gemv_config* cfg);

/* Bytes of workspace dk_w4a16_gemv needs for this shape and config (0 when
 * none).  Replaces the binding's per-call torch::zeros({B,M}) fp32 workspace
 * (bindings.cpp:63-68); contents need no initialisation. */
DK_API size_t dk_w4a16_workspace_bytes(int M, int K, int B, const dk_gemv_config* cfg);

/* y = x . dequant(W)^T.  Replaces decode_kernel::w4a16_gemv
 * (gemv_w4a16.h:34-36, gemv_w4a16.cu:568-591) together with the argument
 * checks of bindings.cpp:10-48.  M, B == 0 is a no-op; K == 0 writes zeros.
 * cfg may be NULL (defaults). */
DK_API dk_status dk_w4a16_gemv(const int32_t* packed, const uint16_t* scales, const uint16_t* x,
                        uint16_t* y, int M, int K, int B, const dk_gemv_config* cfg,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Split-K (version 4) GEMV that allocates nothing and takes no workspace.
 * No counterpart in the reference.  It is for callers that cannot allocate
 * device memory where they call the GEMV -- inside an allocator callback, in
 * a runtime that hands out every buffer itself, or in code that must not
 * touch the allocator on the decode path -- yet still want the split-K
 * kernel.  Its scratch is one fixed buffer of DK_NOALLOC_SCRATCH_BYTES
 * (8 MiB) compiled into the library, held on every GPU that loads the library
 * until the process exits; the caller passes only inputs and outputs.
 *  - Problems whose split-K workspace (dk_w4a16_workspace_bytes with
 *    version 4) exceeds the buffer return DK_ERR_WORKSPACE.  Batches run in
 *    passes of up to 8 rows, so the need is the arrival counters
 *    (ceil(M/16) * 4 bytes, rounded up to 256) plus M * (K/128) * min(B, 8)
 *    * 4 bytes: about M * K <= 268M weights at B = 1, and M * K <= 33M
 *    weights at B >= 8 (M x K = 8176 x 4096 fits, 8192 x 4096 does not).  A split
 *    that clamps to 1 (K = 128) needs no scratch at all.
 *  - The first call on a device looks up the buffer's device address with that
 *    device current; make that first call before any stream capture.  The
 *    address is kept for the life of the process: the library must not be
 *    used across a cudaDeviceReset (or any destruction of the device's
 *    primary context), which may reload the module elsewhere.
 *  - All calls share the one buffer per device: calls that can overlap on the
 *    GPU (different streams without ordering) race and must not be issued.
 *    Each call clears what has to start at zero.
 * Same results, bit for bit, as dk_w4a16_gemv with version 4. */
#define DK_NOALLOC_SCRATCH_BYTES (8u << 20)
DK_API dk_status dk_w4a16_gemv_splitk_noalloc(const int32_t* packed, const uint16_t* scales,
                                              const uint16_t* x, uint16_t* y, int M, int K, int B,
                                              int split_k, void* stream);

/* Several weight matrices that share x -- q/k/v, gate/up -- in one launch:
 * y[i] = x . dequant(W_i)^T for i < n (n <= DK_MAX_SEGMENTS), all with the
 * same K; packed[i] int32 [M[i], K/8], scales[i] fp16 [M[i], K/128], y[i] fp16
 * [B, M[i]].  The streaming kernel runs over the matrices' concatenated row
 * tiles, so every output equals, bit for bit, a dk_w4a16_gemv of its matrix
 * with the same config.  Version 5 or the reuse path; no counterpart in the
 * reference, whose caller (w4a16_linear, python/decode_kernel/__init__.py:
 * 62-83) launches one GEMV per matrix. */
#define DK_MAX_SEGMENTS 4
DK_API dk_status dk_w4a16_gemv_multi(int n, const int32_t* const* packed,
                                     const uint16_t* const* scales, const int* M,
                                     uint16_t* const* y, const uint16_t* x, int K, int B,
                                     const dk_gemv_config* cfg, void* stream);

/* The gate/up pair of a gated MLP with its SiLU-mul epilogue in one launch:
 * h[b, m] = silu(g) * u with g = x . dequant(W_gate)^T, u = x . dequant(W_up)^T
 * (both [M, K]; h fp16 [B, M]).  The roundings are those of the unfused
 * sequence -- g and u as fp16 GEMV outputs (bit for bit dk_w4a16_gemv),
 * silu(g) = g / (1 + exp(-g)) in fp32 rounded to fp16, the product in fp32
 * rounded to fp16 -- so h equals silu(gemv(W_gate, x)) * gemv(W_up, x)
 * computed elementwise in fp16.  Version 5 or the reuse path.  The caller side
 * of the reference's w4a16_linear (python/decode_kernel/__init__.py:62-83)
 * makes two GEMV calls and an elementwise op for this. */
DK_API dk_status dk_w4a16_gemv_silu_mul(const int32_t* packed_gate, const uint16_t* scales_gate,
                                        const int32_t* packed_up, const uint16_t* scales_up,
                                        const uint16_t* x, uint16_t* h, int M, int K, int B,
                                        const dk_gemv_config* cfg, void* stream);

/* ------------------------------------------------------------------------
 * Sharded GEMV across the GPUs of one node (one process per GPU).  No
 * counterpart in the reference, which is single-GPU; these serve the
 * row-parallel (output rows split, results all-gathered) and K-parallel
 * (reduction split, partials summed) layouts, with the exchange fused into
 * the GEMV: every CTA stores its results straight into every rank's buffer
 * over NVLink peer memory.  Row-parallel: each CTA then marks its arrival
 * slot in every rank's slot array with the call's sequence number (one
 * release store per rank), and a rank may read the gathered result once all
 * world * grid slots of its own array carry that number.  K-parallel: each
 * partial travels with the call's sequence number in one 64-bit word, and
 * the sum polls the words themselves (no slots, no separate wait).  All
 * ranks must run on the same GPU model (the grid is derived from the shape
 * and the SM count).
 *
 * Two buffer sets, used in turn.  A rank that has finished call e may store
 * call e+1's results into a slower rank's buffer while that rank still reads
 * call e's gathered result, and a K-parallel word of call e+1 may replace
 * the call-e word before that rank's sum has read it (that sum then waits
 * until its bound runs out).  So every rank keeps two sets of `bufs` (and
 * two dk_shard_group values that differ only in `bufs`; `slots` and `seq`
 * are shared) and consecutive sharded calls alternate between them: set
 * e % 2 for call e.  A set may be written again only by call e+2, i.e.
 * after this rank's wait (dk_shard_wait, DK_FLAG_SHARD_WAIT) or sum
 * (dk_shard_reduce) of call e+1 -- which cannot complete before every rank
 * has finished reading call e's set.  decode_kernel.sharded.PeerBuffers
 * keeps the two sets and alternates them (PeerBuffers.begin()).
 * ------------------------------------------------------------------------ */
#define DK_MAX_SHARDS 8
#define DK_SHARD_SLOTS 256 /* arrival slots per rank and call, >= any grid */
typedef struct dk_shard_group {
  int rank;                        /* this process's rank, 0..world-1 */
  int world;                       /* number of ranks, 1..DK_MAX_SHARDS */
  void* bufs[DK_MAX_SHARDS];       /* every rank's result buffer, mapped here */
  unsigned* slots[DK_MAX_SHARDS];  /* every rank's arrival slots, mapped here:
                                    * unsigned [DK_MAX_SHARDS][DK_SHARD_SLOTS],
                                    * zero before the first call */
  unsigned* seq;                   /* this rank's own unsigned[4] in device
                                    * memory, zero before the first call:
                                    * [0] sharded calls completed on this group,
                                    * [1] CTAs per rank of the last row-parallel
                                    * call, [2] blocks of the running K-parallel
                                    * sum done.  Kept on the device so captured
                                    * graphs replay. */
} dk_shard_group;

/* Row-parallel shard: this rank holds rows [row0, row0 + M_shard) of an
 * [M_total, K] weight (packed [M_shard, K/8], scales [M_shard, K/128]); x is
 * the full fp16 [B, K].  Every rank's bufs[g] is fp16 [B, M_total]; this call
 * writes columns [row0, row0 + M_shard) of all of them.  B <= 32, version 5
 * (cfg->version must be 5; DK_FLAG_PDL is honoured). */
DK_API dk_status dk_w4a16_gemv_rowshard(const int32_t* packed, const uint16_t* scales,
                                        const uint16_t* x, int M_shard, int row0, int M_total,
                                        int K, int B, const dk_shard_group* group,
                                        const dk_gemv_config* cfg, void* stream);

/* Row-parallel shard with the gather fused in, for ranks on separate GPUs
 * running at once, B <= 8 (DK_ERR_UNSUPPORTED above).  As
 * dk_w4a16_gemv_rowshard, but every output travels as one 64-bit word
 * {the fp16-rounded value as fp32 in the low half, the call's sequence number
 * seq[0] + 1 in the high half} -- the K-parallel words' format -- into every
 * rank's bufs[g] (8-byte aligned, [B, M_total] words, columns row0 ..
 * row0 + M_shard - 1), and the same kernel then gathers the whole width:
 * each CTA polls its share of this rank's words until they carry this call's
 * number and writes them to y, fp16 [B, M_total], and the last CTA advances
 * seq[0].  No release fence, slot array or separate wait (slots may be NULL);
 * the two-set rule above applies.  Bounded like dk_shard_wait.  No
 * counterpart in the reference (single-GPU). */
DK_API dk_status dk_w4a16_gemv_rowshard_gather(const int32_t* packed, const uint16_t* scales,
                                               const uint16_t* x, int M_shard, int row0,
                                               int M_total, int K, int B,
                                               const dk_shard_group* group, uint16_t* y,
                                               const dk_gemv_config* cfg, void* stream);

/* K-parallel shard: this rank holds a group-aligned K slice of an [M, K]
 * weight as its own contiguous packed [M, K_shard/8] and scales
 * [M, K_shard/128]; x points at the slice's first column of the full fp16 x,
 * whose rows are ldx elements apart.  Every rank's bufs[g] (8-byte aligned)
 * holds [world][B][M] 64-bit words {fp32 partial in the low half, the call's
 * sequence number seq[0] + 1 in the high half}; this call writes slot `rank`
 * of all of them.  DK_FLAG_SHARD_WAIT is ignored (nothing to wait for).
 * B <= 32. */
DK_API dk_status dk_w4a16_gemv_kshard(const int32_t* packed, const uint16_t* scales,
                                      const uint16_t* x, int ldx, int M, int K_shard, int B,
                                      const dk_shard_group* group, const dk_gemv_config* cfg,
                                      void* stream);

/* K-parallel shard with the sum fused in: as dk_w4a16_gemv_kshard, and then
 * the same kernel adds the world's partials of its rows -- in rank order, the
 * bits of dk_shard_reduce -- into this rank's fp16 y [B, M] and advances
 * seq[0], so no dk_shard_reduce follows (and a PDL-launched successor already
 * streams its weights during the exchange).  Every CTA polls the peers' words
 * for its own rows, so the ranks' calls must run at the same time on
 * different GPUs: ranks that share a GPU use dk_w4a16_gemv_kshard and
 * dk_shard_reduce.  Up to 8 batch rows the sum runs inside the GEMV; with 9..32
 * this call enqueues the GEMV and then dk_shard_reduce (two launches, the same
 * bits).  Bounded like dk_shard_reduce.  No counterpart in the reference
 * (single-GPU). */
DK_API dk_status dk_w4a16_gemv_kshard_sum(const int32_t* packed, const uint16_t* scales,
                                          const uint16_t* x, int ldx, int M, int K_shard, int B,
                                          const dk_shard_group* group, uint16_t* y,
                                          const dk_gemv_config* cfg, void* stream);

/* Enqueue the wait for the sharded call just made on this group: until every
 * arrival slot of this rank's array carries seq[0] + 1, then seq[0] += 1.
 * Later work on the stream sees what every rank stored.  Bounded: after about
 * 2 s it records the timeout in dk_device_error and lets the stream go on. */
DK_API dk_status dk_shard_wait(const dk_shard_group* group, void* stream);

/* K-parallel finish: y[b, m] = fp16(sum over r = 0..world-1, in that order,
 * of partials[r][b][m]) with partials = this rank's buffer bufs[rank] (the
 * 64-bit words above).  Each word is polled until it carries this call's
 * number, then seq[0] += 1; bounded like dk_shard_wait.  `waited` is kept for
 * compatibility and ignored.  Every rank computes the same bits. */
DK_API dk_status dk_shard_reduce(const dk_shard_group* group, int M, int B, uint16_t* y,
                                 int waited, void* stream);

/* Peer memory for the buffers and counters above: a plain device allocation
 * on the current device (zero-filled), its inter-process handle, and the
 * mapping of another process's handle into this one (CUDA IPC over NVLink). */
#define DK_PEER_HANDLE_BYTES 64
DK_API dk_status dk_peer_alloc(size_t bytes, void** ptr);
DK_API dk_status dk_peer_free(void* ptr);
DK_API dk_status dk_peer_export(const void* ptr, unsigned char* handle);
DK_API dk_status dk_peer_import(const unsigned char* handle, void** ptr);
DK_API dk_status dk_peer_close(void* ptr);

/* STREAM-style HBM probes (gemv_w4a16.h:39-43).  `bytes` must be a multiple
 * of 16 and the pointers 16-byte aligned.  dk_stream_read writes one float
 * partial sum per block (blocks <= 0 picks dk_stream_recommended_blocks). */
DK_API dk_status dk_d2d_copy(const void* src, void* dst, size_t bytes, void* stream);
DK_API dk_status dk_stream_read(const void* src, float* partials, size_t bytes, int blocks,
                         void* stream);
DK_API dk_status dk_stream_write(void* dst, size_t bytes, int blocks, void* stream);
/* gemv_w4a16.cu:602-609, but for the given device (-1 = current) instead of
 * always device 0. */
DK_API int dk_stream_recommended_blocks(int device);

/* Stamp written by the GEMV kernel that ran last on `device` (-1 = current):
 * 0..5 for versions 0..5, 10+w for version 1 with w>1 warps per row, 15 for
 * the batch weight-reuse path; -1 if none has run, and -1 when the last GEMV
 * call on that device launched nothing (arguments rejected, empty problem,
 * failed launch) -- the result of the reference's reset of the stamp before
 * every launch (gemv_w4a16.cu:553-557), kept here on the host so that no copy
 * sits between PDL-chained GEMVs on the stream.  Synchronises the device
 * first, like gemv_w4a16.cu:559-564. */
DK_API int dk_last_kernel_stamp(int device);

/* Device-side error word of `device` (-1 = current): 0, or 1 when a bounded
 * wait inside a kernel ran out.  Synchronises the device; clears the word
 * when `clear` is non-zero.  (No counterpart in the reference.) */
DK_API int dk_device_error(int device, int clear);

/* Format helpers on the GPU, bit-exact with python/decode_kernel/quantize.py
 * run on the CPU: quantize_and_pack (:26-51), unpack_to_int (:54-63),
 * dequantize (:66-78).  w is fp32 [M, K]; q is int32 [M, K]. */
#define DK_QUANT_TORCH_CUDA_SCALE 0x1u /* amax * fp32(1/7) instead of amax / 7,
                                        * which is what the same torch code
                                        * computes on a CUDA tensor */
DK_API dk_status dk_quantize_pack(const float* w, int M, int K, int32_t* packed, uint16_t* scales,
                           unsigned flags, void* stream);
DK_API dk_status dk_unpack_to_int(const int32_t* packed, int M, int K, int32_t* q, void* stream);
DK_API dk_status dk_dequantize(const int32_t* packed, const uint16_t* scales, int M, int K, float* w,
                        void* stream);

/* Human-readable text for a status; the CUDA error behind the last
 * DK_ERR_LAUNCH / DK_ERR_CUDA on this thread. */
DK_API const char* dk_status_string(dk_status s);
DK_API const char* dk_last_cuda_error(void);
/* Library version and the architecture it was compiled for ("sm_100a"). */
DK_API const char* dk_version(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* DK_W4A16_H_ */
