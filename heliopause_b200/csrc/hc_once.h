// hc_once.h -- one-time set-up per device, for the kernel launchers.
//
// Kernel attributes (the dynamic shared-memory limit, the shared-memory
// carveout) belong to the device that is current when they are set.  One
// process may drive several devices (hpc_device_init selects the device per
// host thread), so a launcher records, one bit per device, where its set-up
// has succeeded, rather than a single process-wide flag.
//
// Host-only and free of CUDA types, so the logic is testable without a GPU.
#pragma once

#include <atomic>
#include <cstdint>

namespace hc {

// Runs set() unless `done` already holds the bit of `device`, and sets that
// bit when set() returns Err(0) (success); a failed set-up is retried by the
// next call.  Two threads on one device may both run set(), so set() must be
// idempotent (setting an attribute twice is).  Devices outside 0..63 have no
// bit: set() runs on every call.
template <class Err, class F>
Err once_per_device(std::atomic<uint64_t>& done, int device, F&& set) {
  const bool tracked = device >= 0 && device < 64;
  const uint64_t bit = tracked ? (uint64_t(1) << device) : 0;
  if (tracked && (done.load(std::memory_order_acquire) & bit)) return Err(0);
  const Err e = set();
  if (tracked && e == Err(0)) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

}  // namespace hc
