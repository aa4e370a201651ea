// hc_noalloc.cu -- hpc_lm_head_topk_noalloc: the fused LM head + top-k with
// no device allocation inside the call.
//
// hpc_lm_head_topk takes its scratch (the Q8_K activation workspace and the
// per-CTA candidate lists) from cudaMallocAsync on every call.  Callers that
// may not allocate while they serve -- all of HBM handed to weights and the KV
// pool up front, stream-ordered memory pools unavailable, or no allocator
// calls allowed on the decode path -- use this entry point instead.  Its
// scratch is g_lmhead_scratch below: one file-scope device array of
// HPC_NOALLOC_SCRATCH_BYTES per device.
//
//   * The array is shared by every call on a device.  Two calls whose work
//     overlaps in time (different streams, or different host threads) race
//     on it; callers serialize them (one stream, or an event between them).
//   * After a call the array holds that call's Q8_K activations (front) and
//     its per-CTA candidate keys (behind them).  Nothing in it needs to start
//     at zero: the quantize kernel writes the whole workspace, and the LM
//     head kernel clears each candidate slot before filling it.
//   * A call whose scratch would exceed the array returns HPC_ERR_SHAPE
//     with the byte counts in hpc_last_error().
//   * The first call on each device looks the array's address up with
//     cudaGetSymbolAddress (and the launches behind it set their kernel
//     attributes on first use); make that first call outside any stream
//     capture.
// The kernels launched are the fused LM head of hpc_lm_head_topk (per-warp
// candidate lists over the weight stream, then the merge) for every width,
// in the reference's f32 order, so the results equal hpc_lm_head_topk's.
#include <cstdio>
#include <mutex>

#include "../../include/heliocuda.h"
#include "hc_common.cuh"
#include "hc_internal.h"
#include "hc_kernels.cuh"
#include "hc_lmhead.cuh"

static_assert(HPC_NOALLOC_SCRATCH_BYTES % 256 == 0, "scratch size is a multiple of the carve alignment");

static __device__ __align__(256) unsigned char g_lmhead_scratch[HPC_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;

// Address of g_lmhead_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return hpc_cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return hpc_fail(HPC_ERR_CUDA, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_lmhead_scratch);
    if (e != cudaSuccess) return hpc_cuda_fail(e, "cudaGetSymbolAddress(lm head scratch)");
    addr[dev] = p;
  }
  *out = addr[dev];
  return HPC_OK;
}

}  // namespace

extern "C" int hpc_lm_head_topk_noalloc(hpc_weight h, const float* d_hidden, size_t hidden_len, size_t input_size,
                                        size_t column_count, size_t k, int32_t id_offset, float softcap,
                                        int32_t* d_ids, float* d_vals, void* stream) {
  if (hidden_len != input_size * column_count) return hpc_fail(HPC_ERR_SHAPE, "hidden length %zu", hidden_len);
  size_t cb = 0;
  int rc = hpc_lm_head_candidates_bytes(h, column_count, k, &cb);  // validates handle, shape, k
  if (rc != HPC_OK) return rc;
  // the fused path (per-warp candidate lists, reference order) for every
  // width: its candidates are the smallest
  cb = hc_lm_head_fused_candidates_bytes(h, column_count, k);
  size_t head_input = 0;
  rc = hpc_weight_info(h, nullptr, &head_input, nullptr, nullptr);
  if (rc != HPC_OK) return rc;
  if (head_input != input_size)
    return hpc_fail(HPC_ERR_SHAPE, "LM head input size %zu vs %zu", head_input, input_size);
  if (column_count == 0) return HPC_OK;
  if (!d_hidden || !d_ids || !d_vals) return hpc_fail(HPC_ERR_ARG, "null pointer");
  const size_t qb = hc::q8buf_bytes(int(input_size), int(column_count));
  if (qb + cb > size_t(HPC_NOALLOC_SCRATCH_BYTES))
    return hpc_fail(HPC_ERR_SHAPE,
                    "lm head scratch of %zu bytes (Q8_K %zu + candidates %zu) exceeds the static %u-byte scratch",
                    qb + cb, qb, cb, unsigned(HPC_NOALLOC_SCRATCH_BYTES));
  void* ws = nullptr;
  rc = scratch_address(&ws);
  if (rc != HPC_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  hc::Q8Buf q = hc::q8buf_carve(ws, int(input_size), int(column_count));
  cudaError_t e = hc::launch_q8k_quantize(d_hidden, int(input_size), int(column_count), q, nullptr, nullptr, nullptr,
                                          st);
  if (e != cudaSuccess) return hpc_cuda_fail(e, "quantize launch");
  return hc_lm_head_topk_q8_order(h, ws, qb, input_size, column_count, k, id_offset, static_cast<char*>(ws) + qb, cb,
                                  softcap, d_ids, d_vals, nullptr, true, st, true);
}
