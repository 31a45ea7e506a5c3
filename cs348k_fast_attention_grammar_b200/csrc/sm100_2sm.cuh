// Two-SM (cta_group::2) forms for a cluster of two CTAs on an SM pair: the
// even CTA (rank 0) issues tcgen05.mma with M = 256 whose A operand is split
// by rows and B by columns across the two CTAs' shared memory (same offsets),
// and each CTA's TMEM receives its 128 rows of D.  No multicast loads: each
// CTA loads its own operand halves; their completion is counted on the rank-0
// CTA's mbarrier.
#pragma once

#include <cstdint>

namespace fa {

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// All threads of both CTAs; orders shared-memory writes (barrier init) before
// any access from the other CTA.
__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n"
      "barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// Whole-warp, the same warp in both CTAs, the same destination offset.
__device__ __forceinline__ void tmem_alloc_2sm(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_2sm() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_2sm(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T over the CTA pair (issued by rank 0 only).
__device__ __forceinline__ void mma_ss_2sm(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrive once on the mbarrier at offset `bar` of every CTA in `cta_mask` when
// all earlier cta_group::2 MMAs of this thread have completed.
__device__ __forceinline__ void mma_commit_2sm_mc(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar), "h"(cta_mask)
      : "memory");
}
__device__ __forceinline__ void mma_commit_2sm(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 2-D TMA tile load into this CTA's shared memory whose completed bytes are
// counted on the rank-0 CTA's mbarrier at the same offset (bit 24 of a
// shared::cluster address selects the CTA of the pair).
__device__ __forceinline__ void tma_load_2d_2sm(uint32_t dst, const void* map, uint32_t bar,
                                                int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(map), "r"(bar & 0xFEFFFFFFu), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// Arrive on the mbarrier at offset `bar` of CTA `cta` of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar, uint32_t cta) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(bar), "r"(cta));
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote)
               : "memory");
}

}  // namespace fa
