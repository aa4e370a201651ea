// hc_decode.cuh -- launchers of the decoder-math kernels (hc_decode.cu).
#pragma once
#include "hc_common.cuh"

namespace hc {

constexpr int ATT_CHUNK = 64;    // KV tokens per attention CTA (context must be a multiple, <= 4096)
constexpr int ATT_THREADS = 256;

cudaError_t launch_embed(const uint8_t* w, int type, int nb, int vocab, const int32_t* ids, float* hidden, int M, int D,
                         double scale, int* err, cudaStream_t st);
cudaError_t launch_norm_quant(bool resid, const float* x, float* x_out, const float* y, const float* w_post,
                              const float* w_pre, double eps, int M, int D, const Q8Buf& q, float* n_out,
                              cudaStream_t st);
// Dynamic shared memory of one attention CTA for M tokens (staged K/V rows,
// queries, scores), and the most the attention kernels are allowed.
size_t attn_smem_bytes(int M, int H, int KVH);
constexpr size_t ATT_MAX_SMEM = 220 * 1024;
// Attention over the raw q (and, in an own-KV layer, raw k/v) projections of
// M tokens: QK-norm + RoPE of the queries and of this step's K/V rows (written
// to kc/vc), split-KV partials into part_m/part_l/part_o for
// launch_attn_combine.
cudaError_t launch_attention(const float* q, const float* kraw, const float* vraw, const float* qnw, const float* knw,
                             const double* cos_t, const double* sin_t, double eps, bool own_kv, float* kc, float* vc,
                             const int32_t* pos, int M, int H, int KVH, int cap, float scale, float* part_m,
                             float* part_l, float* part_o, int* err, cudaStream_t st);
cudaError_t launch_attn_combine(const float* part_m, const float* part_l, const float* part_o, const int32_t* pos,
                                int M, int H, int KVH, int cap, const Q8Buf& q, float* attn_out, cudaStream_t st);
// The same attention in the reference's exact f32 order (hc_attx.cu):
// scores, softmax and the p.v chains over the keys in order, writing the
// TS-f16-cast output out16 [M][H][256] (the O projection's input before its
// Q8_K quantization).  scratch: attx_scratch_floats(M, H, cap) floats.
size_t attx_scores_smem_bytes(int M, int H, int KVH);
size_t attx_scratch_floats(int M, int H, int cap);
cudaError_t launch_attention_exact(const float* q, const float* kraw, const float* vraw, const float* qnw,
                                   const float* knw, const double* cos_t, const double* sin_t, double eps, bool own_kv,
                                   float* kc, float* vc, const int32_t* pos, int M, int H, int KVH, int cap,
                                   float scale, float* scratch, float* out16, cudaStream_t st);
// cos/sin rows of the tokens at `pos` gathered from the model's table
// [positions][half] (computed on the host, see hc_model.cu); positions at or
// past table_rows are computed on the device.
cudaError_t launch_rope_gather(const int32_t* pos, int M, int half, const double* cos_tab, const double* sin_tab,
                               int table_rows, double theta_scale, double* cos_t, double* sin_t, cudaStream_t st);
// Launches of at least GEGLU_WIDE_MIN_COLS columns (prefill) take a warp per
// 256-block; narrower ones a thread per element, which spreads the f64
// GELU of a decode step over more threads.
constexpr int GEGLU_WIDE_MIN_COLS = 16;
cudaError_t launch_geglu_quant(const float* gate, const float* up, int M, int F, const Q8Buf& q, float* act_out,
                               cudaStream_t st);

// Prefill (many tokens at consecutive positions): QK-norm/RoPE of every
// token's queries into qh [M][H][256] and its K/V rows into the cache, then
// causal attention writing the Q8_K records of the output projection's input.
cudaError_t launch_prefill_qkv_post(const float* q, const float* kraw, const float* vraw, const float* qnw,
                                   const float* knw, const double* cos_t, const double* sin_t, double eps, bool own_kv,
                                   float* kc, float* vc, const int32_t* pos, int M, int H, int KVH, int cap, float* qh,
                                   cudaStream_t st);
cudaError_t launch_prefill_attention(const float* qh, const float* kc, const float* vc, const int32_t* pos, int M,
                                     int H, int KVH, int cap, const Q8Buf& qo, float* attn_out, cudaStream_t st);
// The split form: nsplit = prefill_attn_splits(cap, largest position) splits
// of the key window per query tile, partials [M][H][nsplit] (+ [256] for
// part_o), then the merge (f16 cast + Q8_K, as launch_prefill_attention).
int prefill_attn_splits(int cap, int max_pos);
cudaError_t launch_prefill_attention_split(const float* qh, const float* kc, const float* vc, const int32_t* pos,
                                           int M, int H, int KVH, int cap, int nsplit, float* part_m, float* part_l,
                                           float* part_o, const Q8Buf& qo, float* attn_out, cudaStream_t st);

}  // namespace hc
