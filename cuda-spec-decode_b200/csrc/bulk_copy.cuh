// Bulk-copy (TMA) and mbarrier primitives for sm_100a, as inline PTX.
//
// cp.async.bulk moves a contiguous, 16-byte-aligned range from global memory
// into this CTA's shared memory and completes its byte count on an mbarrier;
// consumers wait on the barrier's phase parity. No multicast form is used.
// Every wait is bounded (kWaitLimitNs on %globaltimer): a caller that times
// out records kStatusTimeout and returns instead of spinning forever.
#pragma once

#include <cstdint>

#include "specdec_common.cuh"

namespace specdec {

constexpr int kStatusTimeout = 5;              // equals SPECDEC_ERR_CUDA in include/specdec.h
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async proxy (the copy engine).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (bulk copy) writes to the same buffer.
__device__ __forceinline__ void fence_proxy_async_smem() {
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
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the phase with the given parity to complete; false after the limit.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

// Releases a stage slot as soon as the calling warp's values are in
// registers, before the arithmetic on them: `dep` is computed from every
// value the lane loaded from the stage (its maximum), and it is an operand of
// both the warp barrier and the arrive, so no lane reaches the barrier -- and
// lane 0 does not arrive -- before its shared-memory loads have returned. The
// producer then refills the slot while the warp works from registers, which
// keeps more of the ring's bytes in flight.
__device__ __forceinline__ void release_stage(uint64_t* empty, float dep) {
  asm volatile("bar.warp.sync %0;" ::"r"(kFullMask), "f"(dep) : "memory");
  if ((threadIdx.x & 31) == 0)
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(empty)), "f"(dep) : "memory");
}

// Bulk copy global -> this CTA's shared memory, completing `bytes` on `bar`.
// src and dst 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace specdec
