// hc_lmhead.cuh -- LM head + top-k launch parameters.
#pragma once
#include "hc_kernels.cuh"

namespace hc {

constexpr int TOPK_MAX = 64;           // TOPK_MAX of runner/webgpu/dispatch.ts:906

struct LmHeadParams {
  GemvParams g;        // seg[0] is the LM-head weight; ksplit = 1, bpc = nb
  int k;               // candidates per column, 1..TOPK_MAX
  int id_offset;       // global vocabulary id of local row 0 (row-sharded heads)
  uint64_t* cand;      // [col][grid][k] keys
  size_t cand_col_stride;
};

int lmhead_grid(int ntiles);
// Candidates per CTA per column: the CTA's merged list of k.
constexpr int LMHEAD_LISTS = 1;
cudaError_t launch_lmhead_topk(const LmHeadParams& P, int grid, cudaStream_t stream);
// Tensor-core LM head + top-k for 3..8 columns (one launch, persistent
// grid of lmhead_mma_grid CTAs, one candidate list per CTA per column).
int lmhead_mma_grid(int ntiles);
cudaError_t launch_lmhead_mma(LmHeadParams& P, int grid, cudaStream_t stream);
// Tensor-core LM head (inputs of >= TC_MIN_COLS columns): the logits are
// written to scratch by launch_gemm_tc, then reduced to candidates in chunks
// of LOGITS_CHUNK_ROWS rows per column.
constexpr int LOGITS_CHUNK_ROWS = 2048;
cudaError_t launch_logits_topk(const float* logits, int rows, int cols, int k, int32_t id_offset, uint64_t* cand,
                               size_t col_stride, cudaStream_t stream);
cudaError_t launch_topk_merge(const uint64_t* cand, int n, size_t col_stride, int group, size_t group_stride, int cols,
                              int k, float softcap, int32_t* ids, float* vals, uint64_t* keys_out,
                              cudaStream_t stream);

}  // namespace hc
