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
