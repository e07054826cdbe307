// objb_tc.cuh -- the sm_100a tensor-core building blocks (tcgen05 / TMEM) used
// by the grouped multi-token contraction: tensor-memory allocation, shared
// memory matrix descriptors for K-major operands without swizzle, the
// kind::i8 MMA, its commit to an mbarrier and 32x32b tensor-memory loads.
//
// Operand layout in shared memory (K-major, SWIZZLE_NONE): "core matrices" of
// 8 rows x 16 bytes stored as 128 contiguous bytes (row r at byte 16 r);
// the core matrix of row group g and 16-byte K chunk c of a tile with KC
// chunks per row sits at (g * KC + c) * 128.  In the descriptor, the leading
// byte offset is the distance between K-adjacent core matrices (128) and the
// stride byte offset between row-adjacent groups (KC * 128).
#pragma once

#include <cstdint>

namespace objb {
namespace dev {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// UMMA shared-memory descriptor (version 1, base offset 0, no swizzle).
__device__ __forceinline__ uint64_t umma_desc_kmajor(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  return d;
}

// One warp allocates `ncols` (a power of two >= 32) tensor-memory columns;
// the base address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols));
}

// The MMA-issuing forms below are executed by every lane of a converged
// warp with warp-uniform operands; the lane elect.sync picks (the same lane
// every time the whole warp is active) issues.  Issued this way a small MMA
// (N <= 96) costs about 60 cycles of issue, against about 100 from a lone
// thread of a diverged warp.

// D[tmem] (=|+=) A x B^T for one K step (32 bytes of int8).
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u));
}

// Arrives on `bar` when every MMA the elected lane issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_addr(bar))
      : "memory");
}

// ---- CTA pairs (cta_group::2): a cluster of two CTAs on two SMs shares
// each MMA (M = 256: 128 rows of A from each CTA's shared memory, N / 2 rows
// of B from each), issued by the even CTA; D lands in each CTA's tensor
// memory (its 128 rows, all N columns).  Allocation and release are
// collective: one warp of each CTA.  Measured on B200: an M256 N48..96 K32
// kind::i8 MMA issues in ~31-37 cycles, against ~170-230 for an M128 one
// from a single CTA.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols));
}
__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, 0, 0;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc));
}
// Arrives on `bar` in both CTAs of the pair when every MMA issued before has completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of both CTAs must reach it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive (release at CTA scope) on the barrier at the same shared-memory
// offset in CTA `rank` of this cluster.  For the operands of a cta_group::2
// MMA in this CTA's shared memory: A rows that its threads wrote (fenced to
// the async proxy before the arrival; only this SM's tensor core reads them)
// and a B half that a bulk copy wrote (its completion observed on a local
// barrier before the arrival).  A release at cluster scope costs the
// arriving thread ~800 cycles.
__device__ __forceinline__ void mbar_arrive_cta(const uint64_t* bar, uint32_t rank) {
  asm volatile(
      "{\n\t.reg .b32 ra;\n\tmapa.shared::cluster.u32 ra, %0, %1;\n\t"
      "mbarrier.arrive.release.cta.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_addr(bar)),
      "r"(rank)
      : "memory");
}
// The same with relaxed semantics: for a barrier that only orders tensor-
// memory accesses, which the tcgen05 fences around it order.
__device__ __forceinline__ void mbar_arrive_cta_relaxed(const uint64_t* bar, uint32_t rank) {
  asm volatile(
      "{\n\t.reg .b32 ra;\n\tmapa.shared::cluster.u32 ra, %0, %1;\n\t"
      "mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_addr(bar)),
      "r"(rank)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 4 / 8 / 16 consecutive 32-bit columns of this warp's 32 tensor-memory lanes.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// The same with two 16-bit columns per register (.pack::16b: the low 16 bits
// of column 2i in bits 0-15, of column 2i + 1 in bits 16-31): 4 / 8 columns.
__device__ __forceinline__ void tmem_ld2_pack16(uint32_t taddr, uint32_t& r0, uint32_t& r1) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.pack::16b.b32 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld4_pack16(uint32_t taddr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                uint32_t& r3) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.pack::16b.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace dev
}  // namespace objb
