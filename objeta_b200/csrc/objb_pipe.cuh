// objb_pipe.cuh -- sm_100a device helpers: mbarriers, 1-D bulk TMA copies
// (cp.async.bulk, no multicast) and bounded waits.
//
// Every wait in this library is bounded: after kMaxSpins failed polls the
// waiting thread records an error code in the caller's error word and gives
// up, so a kernel can never hang the GPU.  Nothing here uses cluster
// multicast; every bulk copy reads this GPU's own memory.
#pragma once

#include <cstdint>

namespace objb {
namespace dev {

// Error codes written to the per-device error word by bounded waits.
constexpr unsigned kErrFullWaitTimeout = 1u;
constexpr unsigned kErrEmptyWaitTimeout = 2u;
constexpr unsigned kErrDrainTimeout = 4u;
constexpr unsigned kErrBadExpertId = 8u;
constexpr unsigned kErrMisaligned = 16u;
constexpr unsigned kErrNoWideSource = 32u;  // a wide digit block met a program without its float vector

// mbarrier.try_wait may suspend the thread for a hardware time slice, so the
// wall-clock bound is kMaxSpins times that slice (well under a few seconds).
constexpr uint32_t kMaxSpins = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Makes the mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
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

// Bounded wait on phase `parity`.  On timeout ORs `code` into the device
// error word *err and raises the launch's CTA-local abort word *abort
// (shared memory); gives up early when another thread of the CTA has already
// raised *abort.  Returns false in both cases.  The device error word only
// records: it keeps codes of earlier launches until objb_device_error_take,
// so it never cuts a wait short.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* err,
                                                  unsigned code, unsigned* abort = nullptr) {
  for (uint32_t i = 0; i < kMaxSpins; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort && (i & 1023u) == 1023u && *reinterpret_cast<volatile unsigned*>(abort) != 0u) return false;
  }
  if (err) atomicOr(err, code);
  if (abort) *reinterpret_cast<volatile unsigned*>(abort) = 1u;
  return false;
}

// L2 policy for data read exactly once (packed weights): evict first.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 1-D bulk copy global -> shared, completion signalled on `bar` as
// transaction bytes.  Requirements (checked by the host before launch):
// both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Named barrier among `nthreads` threads (consumer warps only).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

}  // namespace dev
}  // namespace objb
