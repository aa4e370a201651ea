// hc_bulk.cuh -- one-shot bulk prefetch of weight units into shared memory.
//
// cp.async.bulk (plain form, one CTA as destination) copies a CTA's weight units from HBM into
// shared memory with completion on one mbarrier.  The copies are issued
// before griddepcontrol.wait, so under programmatic dependent launch the
// whole weight fetch of a small GEMV overlaps the previous kernel.  The wait
// is bounded: after ~2 s of %globaltimer it records a timeout in the
// device status word and returns false, so a broken launch cannot hang.
#pragma once
#include <cstdint>

#include "hc_common.cuh"

namespace hc {

constexpr int DEVICE_ERR_TIMEOUT = 1;
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_wait_parity(uint64_t* bar, uint32_t parity, int* err) {
  const unsigned long long t0 = [] {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
  }();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > WAIT_LIMIT_NS) {
      if (err) atomicExch(err, DEVICE_ERR_TIMEOUT);
      return false;
    }
  }
}

// mbar_wait_parity for waits that are expected to last (a weight unit still
// in flight): every try_wait may suspend the warp for up to SLEEP_HINT_NS
// until the phase completes, so a waiting warp does not take issue slots
// from the warps that are computing (a plain try_wait loop spins).  Same
// bound and status as above.
constexpr unsigned SLEEP_HINT_NS = 1000;
__device__ __forceinline__ bool mbar_wait_parity_sleep(uint64_t* bar, uint32_t parity, int* err) {
  unsigned long long t0 = 0;
  for (int it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(SLEEP_HINT_NS)
        : "memory");
    if (ok) return true;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (it == 0) {
      t0 = t;
    } else if (t - t0 > WAIT_LIMIT_NS) {
      if (err) atomicExch(err, DEVICE_ERR_TIMEOUT);
      return false;
    }
  }
}

// A plain arrival (count 1) on an mbarrier of this CTA.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_u32(bar)) : "memory");
}

// dst, src, bytes: multiples of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 16-byte asynchronous global -> shared copy (cp.async.cg, L2 only) issued
// by one thread; cp_async_wait_all waits for the calling thread's copies.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

}  // namespace hc
