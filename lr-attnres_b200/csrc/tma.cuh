// sm_100a asynchronous-copy helpers: mbarriers, 1-D bulk global->shared copies
// (cp.async.bulk, the TMA engine's untiled form, never multicast), named
// barriers, and bounded waits that report through a device status word
// instead of hanging.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace attnres {

// Bit flags written (atomicOr) by a kernel that gave up waiting. Read and
// reset from the host with attnres_device_status().
enum DeviceStatusBits : unsigned {
  kStatusFullWaitTimeout = 1u,   // consumers waited > kWaitLimitNs for a stage to land
  kStatusEmptyWaitTimeout = 2u,  // producer waited > kWaitLimitNs for a stage to drain
  kStatusDrainTimeout = 4u,      // producer gave up waiting for its own copies on exit
};

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s
// Longest time one try_wait may park the thread in hardware before it returns
// false. Parked threads issue nothing, so a waiting warp leaves the issue slots
// to the warps that have data; the bounded loop still checks the 2 s limit.
constexpr uint32_t kSuspendHintNs = 1000000u;  // 1 ms

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete; false after
// `limit_ns` (default ~2 s).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}

// Programmatic dependent launch: block until the grids this launch depends on
// have completed and their writes are visible (a no-op without the launch
// attribute), then let the next launch on the stream start its CTAs.
__device__ __forceinline__ void pdl_wait_then_release() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Barrier over the first `nthreads` threads of the CTA (named barrier 1).
__device__ __forceinline__ void consumer_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Named barrier 2 that also ORs a predicate over the participating threads.
__device__ __forceinline__ bool consumer_sync_or(int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 2, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred ? 1u : 0u), "r"(nthreads)
      : "memory");
  return r != 0;
}

template <typename T, int VEC>
__device__ __forceinline__ Pack<T, VEC> lds_pack(const T* p) {
  return *reinterpret_cast<const Pack<T, VEC>*>(p);
}

}  // namespace attnres
