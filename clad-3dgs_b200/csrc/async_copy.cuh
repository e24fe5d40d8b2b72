// Bulk (TMA 1D) copies, mbarriers and named barriers for sm_100a, plus the
// bounded waits every pipeline barrier goes through.
//
// Every load here is a plain single-CTA bulk copy from this GPU's own memory:
// each CTA fetches its own tiles, and no copy is shared across a cluster.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace clad3dgs {

// Fault codes OR-ed into the per-module fault word when a wait gives up.
enum FaultCode : unsigned {
  kFaultProducerWait = 1u,   // producer timed out waiting for a tile to be computed
  kFaultConsumerWait = 2u,   // consumers timed out waiting for a full stage
};

// Every wait is bounded: a try_wait sleeps at most kSuspendHintNs (it wakes
// as soon as the phase completes), and a wait gives up after kSpinLimit tries,
// i.e. after at most about five seconds, far longer than any launch here.
constexpr uint32_t kSuspendHintNs = 20000;
constexpr uint32_t kSpinLimit = 1u << 18;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(count)
               : "memory");
}

// Makes initialised barriers visible to the async (bulk copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done != 0;
}

// Waits for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar,
                                                  uint32_t parity) {
  for (uint32_t attempt = 0; attempt < kSpinLimit; ++attempt)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// global -> shared bulk copy; completion is counted in bytes on `bar`.
// dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst_smem, const void* src,
                                          uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem_addr(dst_smem)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// shared -> global bulk copy, tracked by bulk groups.
__device__ __forceinline__ void bulk_store(void* dst, const void* src_smem,
                                           uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::
                   "l"(dst),
               "r"(smem_addr(src_smem)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until at most N committed store groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (bulk store) reads of the same bytes.
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace clad3dgs
