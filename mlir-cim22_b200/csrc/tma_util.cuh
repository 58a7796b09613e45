// tma_util.cuh - shared-memory barrier and bulk-tensor copy helpers for the
// layer kernels (sm_100a): a per-CTA TMA load of an f32 box, completed on an
// mbarrier that is waited on with a time limit.
#pragma once

#include <cuda.h>
#include <cstdint>

namespace cim {
namespace {

__device__ __forceinline__ uint32_t shared_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void barrier_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(shared_addr(bar)), "r"(count));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void barrier_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(shared_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void barrier_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(shared_addr(bar)) : "memory");
}

// Wait for the phase with the given parity, for at most limit_ns of the
// global timer (read once every 32 polls). Returns false when it ran out.
__device__ __forceinline__ bool barrier_wait(uint64_t *bar, uint32_t parity,
                                             uint64_t limit_ns = 2000000000ull) {
  const uint32_t addr = shared_addr(bar);
  uint64_t start = 0;
  for (uint32_t i = 1;; ++i) {
    uint32_t done;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(done)
                 : "r"(addr), "r"(parity)
                 : "memory");
    if (done)
      return true;
    if ((i & 31) == 0) {
      uint64_t now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (start == 0)
        start = now;
      else if (now - start > limit_ns)
        return false;
    }
  }
}

// One f32 from a shared-memory byte address.
__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

// A 4-D tiled bulk-tensor load into this CTA's own shared memory only. The
// innermost coordinate x must be a multiple of 4 floats.
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int x, int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(shared_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(shared_addr(bar)), "r"(x), "r"(y), "r"(z),
      "r"(w)
      : "memory");
}

// A 2-D tiled bulk-tensor store from this CTA's shared memory (the layout
// the map's swizzle describes) to global memory, in the thread's bulk async
// group. The innermost coordinate x must be 16-byte aligned in bytes.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x,
                                             int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::
                   "l"(reinterpret_cast<uint64_t>(map)),
               "r"(shared_addr(src)), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until the thread's committed bulk stores have read their shared
// memory (the source may then be rewritten).
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Wait until the thread's committed bulk stores have completed.
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Make this thread's shared-memory writes visible to the async proxy (TMA).
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

} // namespace
} // namespace cim
