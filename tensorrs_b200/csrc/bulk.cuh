// bulk.cuh -- the bulk-copy pipeline primitives (sm_90+ / sm_100a PTX):
// cp.async.bulk global->shared copies completing on an mbarrier with a
// transaction count, and bounded waits on that mbarrier.
//
// Only the issuing CTA's own shared memory is ever a destination, sources are
// this GPU's global memory, and no copy uses cluster multicast.
//
// Every wait is bounded: a CTA that does not see its own copies land within
// kWaitIters polls records an error in the device's async-error word (read
// by trs_async_error()), waits (again bounded) for the copies it still has in
// flight, and returns.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace trs {

constexpr uint32_t kWaitIters = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// 16-byte asynchronous global->shared copies (cp.async, completion by
// commit / wait groups of the issuing thread; both addresses 16-byte aligned).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
// all but the most recently committed group complete
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes initialised mbarriers visible to the async proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses (and, after
// a barrier, the CTA's) before later async-proxy (bulk copy) writes.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// One bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned)
// from global memory into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Tuning knob: the most time (ns) a try_wait may suspend the thread while the
// phase is incomplete (0: the hardware's own limit).
#ifndef TRS_WAIT_HINT_NS
#define TRS_WAIT_HINT_NS 2000
#endif

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
#if TRS_WAIT_HINT_NS > 0
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"((uint32_t)TRS_WAIT_HINT_NS)
      : "memory");
#else
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
#endif
  return ok != 0;
}

// A plain arrive (count 1) on `bar`.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Waits for phase `parity` of `bar` to complete, at most kWaitIters polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kWaitIters; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// The whole CTA waits for phase `parity` of `bar`: thread 0 polls (bounded)
// and the other threads wait at the barrier, where they take no issue slots;
// the barrier after thread 0's acquiring wait makes the copies' data visible
// to every thread.  Returns false on every thread when the poll ran out.
__device__ __forceinline__ bool cta_wait(uint64_t* bar, uint32_t parity) {
  int failed = 0;
  if (threadIdx.x == 0) failed = mbar_wait(bar, parity) ? 0 : 1;
  return __syncthreads_or(failed) == 0;
}

// Programmatic dependent launch.  launch_dependents: the next grid on the
// stream, if launched with programmatic stream serialization, may be
// scheduled now; wait: in that grid, blocks until the previous grid has
// completed and its memory operations are visible (returns at once when the
// grid was launched without the attribute).
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Error codes in the async-error word (bits).
constexpr int kAsyncWaitTimeout = 1;   // a CTA gave up waiting for its own bulk copies
constexpr int kAsyncPeerTimeout = 2;   // the sum exchange gave up waiting for a peer rank

}  // namespace trs
