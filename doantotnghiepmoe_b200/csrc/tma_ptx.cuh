// PTX wrappers for the asynchronous-copy machinery used by the tensor-core
// GEMMs and the decode weight-tile ring: shared-memory mbarriers with
// transaction counts, and 3D tiled TMA loads into this CTA's own shared
// memory.  Every wait is bounded.
#pragma once

#include <cstdint>

namespace moe {
namespace tma {

// ~2 s at 1.9 GHz: far above any legitimate wait, short enough to end a
// stuck launch with an error status instead of hanging the GPU.
constexpr long long kWaitCycles = 4000000000LL;

__device__ __forceinline__ uint32_t su32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(count) : "memory");
}

// Makes barrier initialisation visible to the async proxy (TMA) before use.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (TMA) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(su32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: false on timeout, or (when abort_flag is given) as soon as
// another role has aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          volatile int *abort_flag,
                                          long long limit = kWaitCycles) {
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (abort_flag && *abort_flag) return false;
    if (clock64() - t0 > limit) return false;
  }
  return true;
}

// Box at (c0, c1, c2) of a 3D tiled tensor map into dst (this CTA's shared
// memory); completion is counted on bar in bytes.  c0 * element size must be
// a multiple of 16 bytes.
__device__ __forceinline__ void load_3d(void *dst, const void *map, uint64_t *bar, int c0, int c1,
                                        int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(su32(dst)),
      "l"(map), "r"(su32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

}  // namespace tma
}  // namespace moe
