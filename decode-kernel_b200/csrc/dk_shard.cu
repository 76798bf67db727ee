// dk_shard.cu -- the exchange side of the sharded GEMV: bounded arrival waits,
// the K-parallel partial reduction, and the peer-memory plumbing (CUDA IPC
// handles, mapped with lazy peer access over NVLink).  The call sequence
// number lives on the device (dk_shard_group::seq), so a captured CUDA graph
// of sharded calls replays correctly.
//
// Row-parallel (dk_w4a16_gemv_rowshard in dk_gemv.cu): the kernel stores its
// rows into every rank's buffer and then, per CTA, release-stores the call's
// sequence number into that CTA's slot of every rank's slot array.  The waits
// read the local slots with acquire semantics at system scope, so everything
// the ranks stored before marking their slots is visible to the work that
// follows on the stream.
//
// K-parallel (dk_w4a16_gemv_kshard): the low-latency exchange.  Every fp32
// partial travels with the call's sequence number in one 64-bit word, so the
// sum polls the words themselves -- no release fence on the writer, no slot
// handshake, no separate wait.
#include <cstring>

#include "dk_device.cuh"
#include "dk_host.h"

namespace dk {
namespace {

// The wait for one more call: every slot of this rank's array must carry
// seq[0] + 1 (seq[1] = CTAs per rank of that call, stored by the GEMV).
__global__ void k_shard_wait(const unsigned* slots, unsigned* seq, int world, int* err) {
  const unsigned epoch = seq[0] + 1;
  const int grid = (int)seq[1];
  wait_slots(slots, DK_SHARD_SLOTS, world, grid, epoch, err);
  if (threadIdx.x == 0) seq[0] = epoch;
}

// y[i] = fp16(sum_r part[r][i]) in ascending r; part is [world][n] of 64-bit
// {value, call number} words stored by every rank's GEMV (this GPU's own
// included).  Each word is polled until it carries this call's number
// (bounded: the clock is checked every 256 polls); the last block to finish
// advances seq[0], which every block read before counting itself done
// (seq[2] counts the blocks).
__global__ void k_shard_sum(const unsigned long long* part, int world, int n, __half* y,
                            unsigned* seq, int* err) {
  const unsigned epoch = *reinterpret_cast<volatile unsigned*>(seq) + 1;
  __shared__ int s_abort;
  if (threadIdx.x == 0) s_abort = 0;
  __syncthreads();
  const uint64_t t0 = globaltimer_ns();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < world; ++r) {
      unsigned long long w = ld_ll_sys(part + (size_t)r * n + i);
      for (unsigned polls = 1; (unsigned)(w >> 32) != epoch; ++polls) {
        if ((polls & 255u) == 0 &&
            (*reinterpret_cast<volatile int*>(&s_abort) || globaltimer_ns() - t0 > kWaitLimitNs)) {
          if (!s_abort) atomicExch(err, kDevWaitTimeout);
          s_abort = 1;
          break;
        }
        w = ld_ll_sys(part + (size_t)r * n + i);
      }
      s = __fadd_rn(s, __uint_as_float((unsigned)w));
    }
    y[i] = __float2half_rn(s);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(seq + 2, 1u) == gridDim.x - 1) {
      seq[2] = 0;
      seq[0] = epoch;
    }
  }
}

}  // namespace
}  // namespace dk

using namespace dk;

static bool group_ok(const dk_shard_group* g) {
  return g && g->world >= 1 && g->world <= DK_MAX_SHARDS && g->rank >= 0 &&
         g->rank < g->world && g->slots[g->rank] && g->seq;
}

extern "C" dk_status dk_shard_wait(const dk_shard_group* group, void* stream) {
  if (!group_ok(group)) return DK_ERR_INVALID_ARG;
  int* err = device_error_address();
  if (!err) return DK_ERR_CUDA;
  k_shard_wait<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(group->slots[group->rank],
                                                                 group->seq, group->world, err);
  return check_launch("k_shard_wait");
}

extern "C" dk_status dk_shard_reduce(const dk_shard_group* group, int M, int B, uint16_t* y,
                                     int waited, void* stream) {
  if (!group_ok(group) || !group->bufs[group->rank] || !y || M < 0 || B < 0)
    return DK_ERR_INVALID_ARG;
  (void)waited;  // the words carry their call number: nothing to wait for first
  const long long n = (long long)M * B;
  if (n > (1ll << 30)) return DK_ERR_UNSUPPORTED;
  if (n == 0) return DK_OK;
  if (reinterpret_cast<uintptr_t>(group->bufs[group->rank]) & 7u) return DK_ERR_INVALID_ARG;
  int* err = device_error_address();
  if (!err) return DK_ERR_CUDA;
  const int threads = 256;
  const int blocks = (int)std::min<long long>((n + threads - 1) / threads, 4ll * sm_count(-1));
  k_shard_sum<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const unsigned long long*>(group->bufs[group->rank]), group->world, (int)n,
      reinterpret_cast<__half*>(y), group->seq, err);
  return check_launch("k_shard_sum");
}

extern "C" dk_status dk_peer_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return DK_ERR_INVALID_ARG;
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  if (e != cudaSuccess) {
    set_cuda_error(e, "dk_peer_alloc");
    if (*ptr) cudaFree(*ptr);
    *ptr = nullptr;
    return DK_ERR_CUDA;
  }
  return DK_OK;
}

extern "C" dk_status dk_peer_free(void* ptr) {
  if (!ptr) return DK_OK;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_cuda_error(e, "dk_peer_free");
    return DK_ERR_CUDA;
  }
  return DK_OK;
}

extern "C" dk_status dk_peer_export(const void* ptr, unsigned char* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == DK_PEER_HANDLE_BYTES, "IPC handle size");
  if (!ptr || !handle) return DK_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) {
    set_cuda_error(e, "dk_peer_export");
    return DK_ERR_CUDA;
  }
  std::memcpy(handle, &h, sizeof(h));
  return DK_OK;
}

extern "C" dk_status dk_peer_import(const unsigned char* handle, void** ptr) {
  if (!handle || !ptr) return DK_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_cuda_error(e, "dk_peer_import");
    *ptr = nullptr;
    return DK_ERR_CUDA;
  }
  return DK_OK;
}

extern "C" dk_status dk_peer_close(void* ptr) {
  if (!ptr) return DK_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    set_cuda_error(e, "dk_peer_close");
    return DK_ERR_CUDA;
  }
  return DK_OK;
}
