// Thread-block-cluster helpers for sm_100a: cluster ids, barriers, mapping a
// shared address into another CTA of the cluster, bulk copies and 4/16-byte
// stores into a cluster CTA's shared memory that complete on its mbarrier
// (none of them multicast), and bounded cluster-scope mbarrier waits.
#pragma once

#include <stdint.h>

#include "tma.cuh"

namespace attnres {

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// this CTA's shared address `a` as seen in cluster CTA `rank`
__device__ __forceinline__ uint32_t map_to_rank(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
// bulk copy of this CTA's shared bytes into a cluster CTA's shared memory,
// completing (complete_tx) on that CTA's mbarrier
__device__ __forceinline__ void bulk_s2cluster(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst),
               "r"(smem_u32(src)), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait on a barrier completed by other CTAs of the cluster
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}
// remote shared-memory stores that complete (complete_tx) on the target CTA's
// mbarrier: the logits (4 bytes) and the credit signals (16 bytes)
__device__ __forceinline__ void st_async_f32(uint32_t dst, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(dst),
               "r"(__float_as_uint(v)), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void st_async_signal(uint32_t dst, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %1, %1, %1}, [%2];" ::"r"(
                   dst),
               "r"(0u), "r"(bar)
               : "memory");
}
}  // namespace attnres
