// peer.cu - peer memory and a device-side barrier for layers whose output
// lanes are split over the GPUs of one node.
//
// Each rank allocates its full layer outputs and a small flag array here,
// exports them as CUDA IPC handles, and maps every other rank's buffers. The
// column-sharded contraction (gemm_tc.cu, launch_signsplit_b16 with peer
// outputs) then writes each rank's lane block into all ranks' outputs over
// NVLink, and cim22_cuda_peer_barrier orders the layers: no collective
// library call sits between two layers. Plain loads and stores only (no
// multicast objects, no TMA on peer memory).
#include "cim_internal.h"

#include <cstring>

namespace cim {
namespace {

static_assert(sizeof(cudaIpcMemHandle_t) == CIM22_IPC_HANDLE_BYTES,
              "the C-ABI handle size must match the runtime's IPC handle");

__device__ __forceinline__ void store_release_sys(int32_t *p, int32_t v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int32_t load_acquire_sys(const int32_t *p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One thread: raise the epoch, publish it to every rank, wait for every
// rank's. The fence makes the stream's earlier writes (the contraction's
// peer stores, ordered before this kernel by the stream) visible system-wide
// before the release stores of the epoch; the acquire loads order the next
// kernel's reads after the peers' writes.
__global__ void peer_barrier_kernel(cim22_peer_flags f, uint64_t limit_ns, int32_t *status) {
  if (threadIdx.x != 0 || blockIdx.x != 0)
    return;
  int32_t *own = f.flags[f.rank];
  const int32_t epoch = own[f.ranks] + 1;
  own[f.ranks] = epoch;
  __threadfence_system();
  for (int p = 0; p < f.ranks; ++p)
    store_release_sys(f.flags[p] + f.rank, epoch);
  const uint64_t start = global_timer_ns();
  for (int q = 0; q < f.ranks; ++q) {
    uint32_t polls = 0;
    while (load_acquire_sys(own + q) < epoch) {
      if ((++polls & 255u) == 0 && global_timer_ns() - start > limit_ns) {
        atomicOr(status, CIM22_STATUS_TIMEOUT);
        return;
      }
    }
  }
}

} // namespace
} // namespace cim

using namespace cim;

extern "C" {

int cim22_cuda_device_alloc(size_t bytes, void **ptr) {
  if (!ptr || bytes == 0) {
    set_last_error("invalid arguments to cim22_cuda_device_alloc");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  *ptr = nullptr;
  if (!cuda_ok(cudaMalloc(ptr, bytes), "cudaMalloc"))
    return CIM22_STATUS_BAD_ARGUMENT;
  if (!cuda_ok(cudaMemset(*ptr, 0, bytes), "cudaMemset")) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  return 0;
}

int cim22_cuda_device_free(void *ptr) {
  if (!ptr)
    return 0;
  return cuda_ok(cudaFree(ptr), "cudaFree") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

int cim22_cuda_ipc_get_handle(const void *base, void *handle) {
  if (!base || !handle) {
    set_last_error("invalid arguments to cim22_cuda_ipc_get_handle");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  cudaIpcMemHandle_t h;
  if (!cuda_ok(cudaIpcGetMemHandle(&h, const_cast<void *>(base)), "cudaIpcGetMemHandle"))
    return CIM22_STATUS_BAD_ARGUMENT;
  std::memcpy(handle, &h, sizeof(h));
  return 0;
}

int cim22_cuda_ipc_open_handle(const void *handle, void **base) {
  if (!handle || !base) {
    set_last_error("invalid arguments to cim22_cuda_ipc_open_handle");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *base = nullptr;
  return cuda_ok(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess),
                 "cudaIpcOpenMemHandle")
             ? 0
             : CIM22_STATUS_BAD_ARGUMENT;
}

int cim22_cuda_ipc_close_handle(void *base) {
  if (!base)
    return 0;
  return cuda_ok(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle") ? 0
                                                                       : CIM22_STATUS_BAD_ARGUMENT;
}

int cim22_cuda_peer_barrier(const cim22_peer_flags *flags, uint64_t limit_ns, int32_t *status,
                            void *stream) {
  if (!flags || !status || flags->ranks < 1 || flags->ranks > CIM22_MAX_PEERS ||
      flags->rank < 0 || flags->rank >= flags->ranks) {
    set_last_error("invalid arguments to cim22_cuda_peer_barrier");
    return CIM22_STATUS_BAD_ARGUMENT;
  }
  for (int p = 0; p < flags->ranks; ++p)
    if (!flags->flags[p]) {
      set_last_error("cim22_cuda_peer_barrier: a rank's flag array is missing");
      return CIM22_STATUS_BAD_ARGUMENT;
    }
  // A plain launch: it starts once the stream's previous kernel has
  // completed, so the contraction's peer stores precede the fence.
  peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(*flags, limit_ns,
                                                                         status);
  return cuda_ok(cudaGetLastError(), "peer barrier launch") ? 0 : CIM22_STATUS_BAD_ARGUMENT;
}

} // extern "C"
