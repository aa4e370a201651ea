// hc_internal.h -- definitions shared by the C-ABI translation units.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/heliocuda.h"

constexpr uint32_t kWeightMagic = 0x48504357u;  // "HPCW"

// A resident weight: GGUF bytes repacked into the tile layout (hc_common.cuh).
struct hpc_weight_s {
  uint32_t magic;
  int type;
  int device;
  size_t input_size;
  size_t row_count;
  size_t rows_pad;
  int nb;
  uint8_t* d_data;
  size_t bytes;
};

inline bool hpc_weight_valid(const hpc_weight_s* h) { return h && h->magic == kWeightMagic && h->d_data; }

// Records a message for hpc_last_error() and returns `code`.
int hpc_fail(int code, const char* fmt, ...);
int hpc_cuda_fail(cudaError_t e, const char* what);

#define HPC_CK(call, what)                                  \
  do {                                                      \
    cudaError_t e_ = (call);                                \
    if (e_ != cudaSuccess) return hpc_cuda_fail(e_, what);  \
  } while (0)

namespace hc {
struct GemvPrologue;
}
// hpc_matmul_q8 with the fused norm prologue (hc_api.cu).
int hc_matmul_q8_prologue(size_t count, const hpc_weight* handles, const void* q8ws, size_t q8_bytes, size_t input_size,
                          size_t column_count, float* const* d_outs, const size_t* out_lens,
                          const hc::GemvPrologue& pro, cudaStream_t st);
// The exact-order matmul with every CTA computing its input (hc_gemvx.cu
// prologue): width 2048, up to 8 columns.
int hc_matmul_q8_exact_prologue(size_t count, const hpc_weight* handles, const void* q8ws, size_t q8_bytes,
                                size_t input_size, size_t column_count, float* const* d_outs, const size_t* out_lens,
                                const hc::GemvPrologue& pro, cudaStream_t st);
// hpc_matmul_q8 with the order chosen: exact = the reference's f32 order
// (every path hpc_matmul_* exposes), or the reordered fast kernels (dp4a /
// tensor-core GEMV) the model's reordered step uses.
int hc_matmul_q8_order(size_t count, const hpc_weight* handles, const void* d_workspace, size_t workspace_bytes,
                       size_t input_size, size_t column_count, float* const* d_outs, const size_t* out_lens,
                       bool exact, cudaStream_t stream);
// hpc_lm_head_topk_q8 with the order chosen (exact: reference-order logits
// for every width below the tensor-core matmul's).
// fused_only: the dp4a LM head with per-warp candidate lists for every
// width, in the exact order (passes of 2 columns) -- the path whose
// candidate buffer (hc_lm_head_fused_candidates_bytes) is the smallest.
int hc_lm_head_topk_q8_order(hpc_weight lm_head, const void* d_workspace, size_t workspace_bytes, size_t input_size,
                             size_t column_count, size_t k, int32_t id_offset, void* d_candidates,
                             size_t candidates_bytes, float softcap, int32_t* d_ids, float* d_vals, uint64_t* d_keys,
                             bool exact, cudaStream_t stream, bool fused_only = false);
size_t hc_lm_head_fused_candidates_bytes(hpc_weight lm_head, size_t column_count, size_t k);
