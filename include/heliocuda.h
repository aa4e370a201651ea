/*
 * heliocuda.h -- C ABI of the B200 (sm_100a) runner for the Heliopause decode
 * hot path: Q4_K/Q6_K dequant-fused GEMV and small-M matmul, the Q6_K LM head
 * with on-GPU top-k, and the pieces of the decode step around them.
 *
 * Conventions
 *   - Plain C types only.  `stream` is a cudaStream_t passed as void*
 *     (NULL = the legacy default stream).  Device pointers are marked d_*.
 *   - Lengths are element counts (bytes for weight buffers), exactly as in
 *     the WASM exports these functions replace.
 *   - Matrices follow the reference layout: a weight has `row_count` output
 *     rows of `input_size` elements; activations are `column_count` columns of
 *     `input_size` floats (x[col*input_size + i]); outputs are
 *     out[col*row_count + row].
 *   - Every call returns a status code.  0..3 are the reference's codes
 *     (packages/engine/wasm-kernels/src/lib.rs:7-10); 4..7 are added for the
 *     GPU.  hpc_last_error() gives a message for the calling thread.
 *   - Calls are stream-ordered and do not synchronize unless noted.
 *   - The library never falls back to the CPU: without a usable device every
 *     call returns HPC_ERR_CUDA.
 */
#ifndef HELIOCUDA_H
#define HELIOCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HPC_OK 0
#define HPC_ERR_SHAPE 1   /* lib.rs:8  ERR_SHAPE */
#define HPC_ERR_HEADS 2   /* lib.rs:9  ERR_HEADS */
#define HPC_ERR_TYPE 3    /* lib.rs:10 ERR_TYPE  */
#define HPC_ERR_CUDA 4    /* CUDA runtime or launch failure */
#define HPC_ERR_TIMEOUT 5 /* a bounded device wait gave up */
#define HPC_ERR_NCCL 6    /* collective failure */
#define HPC_ERR_ARG 7     /* null pointer / invalid handle */

/* Type ids: lib.rs:12-17 and quantizedTypeId (runner/wasm/wasm-kernels.ts:1908-1923). */
#define HPC_TYPE_Q4_K 1
#define HPC_TYPE_Q5_K 2
#define HPC_TYPE_Q6_K 3
#define HPC_TYPE_IQ4_XS 4
#define HPC_TYPE_Q8_0 5
#define HPC_TYPE_Q4_0 6

/* Opaque resident weight (HBM).  Replaces WasmQuantizedWeightHandle
 * (runner/wasm/wasm-kernels.ts:387-397): it owns the uploaded bytes, already
 * repacked into the coalesced tile layout the kernels read. */
typedef struct hpc_weight_s *hpc_weight;

/* Message of the last failing call on this thread ("" if none). */
const char *hpc_last_error(void);

/* ABI version (major << 16 | minor). */
int hpc_version(void);

/* Reads and clears the current device's status word: HPC_ERR_TIMEOUT if a
 * kernel's bounded wait gave up since the last call, else HPC_OK.
 * Synchronizes with the device. */
int hpc_device_error(void);

/* Select the device for subsequent calls on this thread and check it is an
 * sm_100 part.  Replaces prefillWasmExports() instantiation
 * (runner/wasm/wasm-kernels.ts:416-426).  One process may drive several
 * devices, one per host thread.  Each launcher sets its kernel attributes
 * on a device at its first call there; make that first call outside any
 * stream capture. */
int hpc_device_init(int device);

/* Upload a GGUF-layout weight (host bytes) and repack it in HBM.  Only Q4_K
 * and Q6_K are resident on the GPU; other type ids return HPC_ERR_TYPE.
 * Replaces createWasmQuantizedWeightHandle (wasm-kernels.ts:520-574), which
 * copies the bytes and runs hp_prepare_quantized_scales_f32 (lib.rs:157-222).
 * Synchronous. */
int hpc_weight_upload(int type_id, const uint8_t *host_bytes, size_t byte_len, size_t input_size,
                      size_t row_count, hpc_weight *out_handle);

/* Same, from GGUF-layout bytes already in device memory (not modified). */
int hpc_weight_upload_device(int type_id, const void *d_bytes, size_t byte_len, size_t input_size,
                             size_t row_count, void *stream, hpc_weight *out_handle);

/* Replaces releaseWasmQuantizedWeightHandle (wasm-kernels.ts:576-584). */
int hpc_weight_release(hpc_weight handle);

/* Shape and residency of a handle (any out pointer may be NULL). */
int hpc_weight_info(hpc_weight handle, int *type_id, size_t *input_size, size_t *row_count,
                    size_t *device_bytes);

/* Dequantize the resident weight to f32 [row_count][input_size], bit-exact
 * to dequantize_q4_k / dequantize_q6_k (lib.rs:1630-1664, 1709-1744). */
int hpc_weight_dequantize(hpc_weight handle, float *d_out, size_t out_len, void *stream);

/* Q8_K activation quantization of `column_count` columns, bit-exact to
 * quantize_q8_k (lib.rs:1774-1811): d_d[col*(K/256)], d_qs[col*K] (natural
 * element order), d_bsums[col*(K/32)]. */
int hpc_quantize_q8_k(const float *d_in, size_t in_len, size_t input_size, size_t column_count, float *d_d,
                      int8_t *d_qs, int16_t *d_bsums, void *stream);

/* Arithmetic order of the matmul and LM-head entry points below
 * (process-wide).  exact != 0 (the default): every output row dot of fewer
 * than 16 columns is vec_dot_q4_k_q8_k_prepared / vec_dot_q6_k_q8_k_prepared
 * (lib.rs:1924-1968, 2117-2172) in its own f32 order -- eight lane
 * accumulators, block by block -- so results equal the WASM exports bit for
 * bit.  exact == 0: the reordered kernels (dp4a GEMV, tensor-core GEMV and
 * LM head for 3-8 columns), equal to f32 rounding.  16 or more columns run on
 * the tensor cores in either order.  Calls already enqueued keep the order
 * they were made with. */
int hpc_set_matmul_order(int exact);

/* Resident GEMV / small-M matmul with Q8_K activations.
 * Replaces hp_matmul_quantized_prepared_f32 (lib.rs:225-298) as called by
 * matMulQuantizedWasmResident (wasm-kernels.ts:593-646); same validation
 * order and codes.  column_count may be any value >= 1 (processed 8 columns
 * per pass). */
int hpc_matmul_quantized_prepared_f32(hpc_weight handle, const float *d_in, size_t in_len, size_t input_size,
                                      size_t row_count, size_t column_count, float *d_out, size_t out_len,
                                      void *stream);

/* Several resident weights sharing one input, in ONE launch; the input is
 * quantized once.  Replaces hp_matmul_quantized_prepared_multi_f32
 * (lib.rs:302-426) via matMulQuantizedWasmResidentMulti
 * (wasm-kernels.ts:648-749); count is 1..8 here (the reference caps at 4). */
int hpc_matmul_quantized_prepared_multi_f32(size_t count, const float *d_in, size_t in_len, size_t input_size,
                                            size_t column_count, const hpc_weight *handles, float *const *d_outs,
                                            const size_t *out_lens, void *stream);

/* One-shot matmul on HOST buffers: upload, repack, quantize, multiply,
 * download, release.  Replaces hp_matmul_quantized_f32 (lib.rs:41-100) as
 * called by matMulQuantizedWasm (wasm-kernels.ts:416-466).  Synchronous. */
int hpc_matmul_quantized_f32(int type_id, const uint8_t *host_weight, size_t weight_len, const float *host_in,
                             size_t in_len, size_t input_size, size_t row_count, size_t column_count,
                             float *host_out, size_t out_len);

/* Dequantized matmul: every weight row is dequantized bit-exactly and
 * multiplied by each input column with the reference's sequential f32 sum
 * (sum = fround(sum + fround(w * x)) in index order), so outputs equal
 * hp_matmul_dequantized_f32 (lib.rs:103-154) bit for bit.  The reference
 * calls it through matMulDequantizedWasm (wasm-kernels.ts:468-520) for the
 * MTP draft head (runner/wasm/mtp-assistant-runner.ts:156-180).  Same
 * validation order and codes as the WASM export.  One-shot on HOST buffers
 * (upload, multiply, download, release; synchronous): */
int hpc_matmul_dequantized_f32(int type_id, const uint8_t *host_weight, size_t weight_len, const float *host_in,
                               size_t in_len, size_t input_size, size_t row_count, size_t column_count,
                               float *host_out, size_t out_len);

/* Same arithmetic on a resident weight and device buffers, stream-ordered. */
int hpc_matmul_dequantized_prepared_f32(hpc_weight handle, const float *d_in, size_t in_len, size_t input_size,
                                        size_t row_count, size_t column_count, float *d_out, size_t out_len,
                                        void *stream);

/* ---- caller-provided scratch ("workspace") variants ----------------------
 * The activation is quantized once into a workspace the caller allocates
 * (no allocation inside the call, so these can be captured in a CUDA graph),
 * then any number of resident weights consume it.  They split
 * matMulQuantizedWasmResident(Multi) into its two phases: quantize_q8_k
 * (lib.rs:1774) and the per-row dots (lib.rs:264-296). */

/* Workspace bytes for `column_count` columns of `input_size`. */
int hpc_q8_workspace_bytes(size_t input_size, size_t column_count, size_t *out_bytes);

/* Quantize f32 columns into the workspace (Q8_K, bit-exact to lib.rs:1774). */
int hpc_q8_quantize(const float *d_in, size_t in_len, size_t input_size, size_t column_count, void *d_workspace,
                    size_t workspace_bytes, void *stream);

/* Multiply `count` (1..8) resident weights against a quantized workspace in
 * one launch per 8 columns; outputs as hpc_matmul_quantized_prepared_multi_f32. */
int hpc_matmul_q8(size_t count, const hpc_weight *handles, const void *d_workspace, size_t workspace_bytes,
                  size_t input_size, size_t column_count, float *const *d_outs, const size_t *out_lens, void *stream);

/* The tensor-core kind of the >= 16-column Q4_K matmul (prefill, the wide LM
 * head): 0 = mma.sync s8 (default), 1 = tcgen05.mma kind::i8 with the
 * accumulators in tensor memory.  Both compute the same integer block sums
 * and the same f32 combine; results are bit-identical where the mma.sync
 * launch does not split K (it splits launches of fewer than two CTAs per
 * SM in two halves, added atomically).  Process-wide. */
int hpc_set_wide_matmul_kind(int kind);

/* The norm-fused projection of the decode step: the rmsNorm of the residual
 * stream (wasm/layers.ts:161-247 -- optionally after adding the previous
 * projection through its post-norm), quantize_q8_k (lib.rs:1774-1811) and
 * the prepared multi matmul (lib.rs:302-426), with the norms and the
 * quantization computed inside the matmul launch by every CTA:
 *   h = d_y ? x + f32(rmsNorm(y) * w_post) : x     (h stored to d_x_out when d_y)
 *   out_i = W_i . Q8_K(f32(rmsNorm(h) * w_pre))
 * rmsNorm in f64 as the WASM provider computes it.  input_size must be 2048
 * and column_count 1..8 (1..2 under the reordered matmul order);
 * d_x_out must not alias d_x.  The workspace carries the Q8_K geometry as
 * for hpc_matmul_q8. */
int hpc_matmul_rmsnorm_f32(size_t count, const hpc_weight *handles, void *d_workspace, size_t workspace_bytes,
                           size_t input_size, size_t column_count, const float *d_x, const float *d_y,
                           const float *d_w_post, const float *d_w_pre, double eps, float *d_x_out,
                           float *const *d_outs, const size_t *out_lens, void *stream);

/* ---- LM head with on-GPU top-k --------------------------------------------
 * Ordering everywhere: value descending, then vocabulary id ascending
 * (topK, runtime.ts:514-527; betterValue in TOPK_CHUNK_CANDIDATES_WGSL,
 * runner/webgpu/shaders.ts:1591-1650).  k is 1..64 (TOPK_MAX,
 * runner/webgpu/dispatch.ts:906).  Values are the raw logits, or
 * fround(tanh(v/cap)*cap) when softcap > 0, applied after selection as
 * mergeTopCandidates does (runner/webgpu/segment-runner.ts:3773-3794). */

/* Fused Q6_K/Q4_K LM head + top-k on f32 hidden columns (already normed):
 * ids/vals are [column_count][k].  Replaces dispatchOutputTopK
 * (runner/webgpu/segment-runner.ts:3208-3248) and the WASM forwardOutput
 * logits + topK (runner/wasm/layers.ts:381-416).  id_offset is the vocabulary
 * id of the handle's row 0 (row-sharded heads). */
int hpc_lm_head_topk(hpc_weight lm_head, const float *d_hidden, size_t hidden_len, size_t input_size,
                     size_t column_count, size_t k, int32_t id_offset, float softcap, int32_t *d_ids, float *d_vals,
                     void *stream);

/* Candidate-buffer bytes for hpc_lm_head_topk_q8. */
int hpc_lm_head_candidates_bytes(hpc_weight lm_head, size_t column_count, size_t k, size_t *out_bytes);

/* Same on a quantized workspace (hpc_q8_quantize), with a caller-provided
 * candidate buffer; also writes the selected 64-bit keys
 * (orderable(value) << 32 | 0xFFFFFFFF - id) when d_keys != NULL, which is
 * what a row-sharded head all-gathers before hpc_topk_merge_keys. */
int hpc_lm_head_topk_q8(hpc_weight lm_head, const void *d_workspace, size_t workspace_bytes, size_t input_size,
                        size_t column_count, size_t k, int32_t id_offset, void *d_candidates, size_t candidates_bytes,
                        float softcap, int32_t *d_ids, float *d_vals, uint64_t *d_keys, void *stream);

/* Merge gathered keys laid out [group_count][column_count][k] into the
 * global top-k per column (the cross-GPU merge of a row-sharded LM head). */
int hpc_topk_merge_keys(const uint64_t *d_keys, size_t group_count, size_t column_count, size_t k, float softcap,
                        int32_t *d_ids, float *d_vals, void *stream);

/* One token drawn from a candidate list on the device (replaces the host's
 * token_sampling_distribution + sample_next_token, generation.ts:85-165, and
 * the mulberry32-style generator of generation.ts:74-83).  d_ids / d_vals:
 * n (1..1024) candidates sorted by value descending then id ascending, as the
 * top-k entry points write them.  Keeps the first top_k, then the top_p
 * nucleus, then draws from the softmax of value / temperature with the
 * generator advanced once from rng_state (the caller advances its own copy
 * of the stream by one draw); greedy != 0 takes the first candidate and
 * draws nothing.  Writes the token to *d_token and, when d_table != NULL
 * (f32 [table_rows][hidden]), d_table[token][0..hidden) * scale (f64 product
 * rounded to f32) to d_row_out, the next draft step's input embedding; a
 * token outside [0, table_rows) leaves d_row_out untouched.  The exps are
 * the device's f64 exp. */
int hpc_sample_candidates(const int32_t *d_ids, const float *d_vals, size_t n, size_t top_k, double top_p,
                          double temperature, int greedy, uint32_t rng_state, int32_t *d_token, const float *d_table,
                          size_t table_rows, size_t hidden, double scale, float *d_row_out, void *stream);

/* ---- LM head + top-k with no allocation inside the call --------------------
 * No reference counterpart: an addition for callers that may not allocate
 * device memory while they serve (all of HBM handed to weights and the KV
 * pool up front, stream-ordered memory pools unavailable, or no allocator
 * calls allowed on the decode path).  Same arguments, checks and results as
 * hpc_lm_head_topk, which takes its scratch from cudaMallocAsync; this one
 * uses a file-scope device array of HPC_NOALLOC_SCRATCH_BYTES per device:
 *   - a call needing more scratch (Q8_K workspace + candidate lists, e.g.
 *     1.9 MB for 262,144 rows, 8 columns, k = 64) returns HPC_ERR_SHAPE;
 *   - the array is shared by all calls on the device: calls that overlap in
 *     time (other streams or threads) race on it, so serialize them;
 *   - after a call it holds that call's Q8_K activations and candidate keys;
 *     nothing in it needs to start at zero;
 *   - the first call on each device does one-time set-up
 *     (cudaGetSymbolAddress, kernel attributes): make it outside any stream
 *     capture. */
#define HPC_NOALLOC_SCRATCH_BYTES (4u << 20)
int hpc_lm_head_topk_noalloc(hpc_weight lm_head, const float *d_hidden, size_t hidden_len, size_t input_size,
                             size_t column_count, size_t k, int32_t id_offset, float softcap, int32_t *d_ids,
                             float *d_vals, void *stream);

/* ---- resident decoder model: decode / batched verify step ------------------
 * A Gemma-4-style decoder (pre/post RMSNorm sandwich, per-head QK norm, NeoX
 * RoPE, GQA over an fp32 KV cache, GEGLU FFN, tied Q6_K/Q4_K embedding / LM
 * head) kept resident in HBM.  hpc_model_forward runs embedding -> all layers
 * -> output norm -> LM head top-k for token_count consecutive positions in one
 * CUDA-graph launch: the WASM provider's per-token forward
 * (runner/wasm/layers.ts:161-473, forwardOutput :381-416) and the WebGPU
 * batched verify forward (runner/webgpu/segment-runner.ts:1292-1606). */

typedef struct hpc_model_s *hpc_model;

typedef struct {
  int hidden;        /* embeddingLength, multiple of 2048 */
  int heads;         /* query heads */
  int kv_heads;      /* key/value heads (GQA) */
  int head_dim;      /* 256 */
  int ffn;           /* feed_forward_length, multiple of 2048 */
  int vocab;
  int layers;
  int kv_layers;     /* layers [0, kv_layers) own a KV cache; later layers reuse
                        layer kv_layers-1's (kvSourceLayers, engine/src/model.ts:382-388) */
  int context;       /* KV capacity (full attention) */
  int max_tokens;    /* largest token_count per call, 1..8; max_tokens *
                        heads / kv_heads <= 72 (the query vectors one
                        attention CTA stages), else HPC_ERR_SHAPE */
  int top_k;         /* largest top_k per call, 1..64 */
  double rms_eps;
  double rope_theta;
  float final_logit_softcap; /* <= 0: none */
} hpc_model_config;

/* weight slots */
#define HPC_W_Q 0
#define HPC_W_K 1
#define HPC_W_V 2
#define HPC_W_O 3
#define HPC_W_GATE 4
#define HPC_W_UP 5
#define HPC_W_DOWN 6
#define HPC_W_COUNT 7
/* norm slots (f32 weights) */
#define HPC_N_ATTN 0
#define HPC_N_Q 1
#define HPC_N_K 2
#define HPC_N_POST_ATTN 3
#define HPC_N_FFN 4
#define HPC_N_POST_FFW 5
#define HPC_N_COUNT 6
#define HPC_N_OUTPUT 100 /* output_norm (layer ignored) */

int hpc_model_create(const hpc_model_config *config, hpc_model *out_model);
int hpc_model_release(hpc_model model);
/* The model does not own weight handles; they must outlive it. */
int hpc_model_set_weight(hpc_model model, int layer, int slot, hpc_weight weight);
int hpc_model_set_norm(hpc_model model, int layer, int slot, const float *host_values, size_t len);
/* token_embd.weight == output weight (tied): rows are vocabulary ids. */
int hpc_model_set_lm_head(hpc_model model, hpc_weight weight);
/* Arithmetic order of the model's steps.  enable != 0 (the default): every
 * step computes in the reference's own order -- each matmul row dot with the
 * eight f32 lane accumulators of vec_dot_q*_k_q8_k_prepared
 * (lib.rs:1924-1968, 2117-2172), the attention's dots, softmax sum and
 * p.v sums as the sequential f32 chains of hp_gqa_attention_f32
 * (lib.rs:539-654), RoPE angles from host-computed cos/sin -- so its top-k
 * ids and values equal the WASM provider's (runner/wasm/layers.ts:161-473,
 * forwardOutput :381-416) bit for bit.  enable == 0: the reordered kernels
 * (split-KV attention with a combine, norms fused into the GEMVs, the
 * tensor-core GEMV / LM head for 3-8 tokens): faster, equal to the
 * reference only to f32 rounding, which the Q8_K re-quantization of every
 * matmul input amplifies over the layers. */
int hpc_model_set_exact(hpc_model model, int enable);

/* Device pointers of one KV layer's cache, f32: K [context][kv_heads][head_dim]
 * (the layers.ts:887-911 layout) and V [context][kv_heads][head_dim] -- V is
 * token-major like K, the transpose of the reference's [head_dim][kv_heads]
 * [context], so that one token's values are one contiguous row. */
int hpc_model_kv(hpc_model model, int kv_layer, float **d_key, float **d_value);
/* One forward over token_count tokens at the given positions (all device
 * pointers).  Writes top-k ids/values [token_count][top_k] for every position
 * (value desc, id asc; softcap after selection), and the final residual stream
 * [token_count][hidden] when d_hidden_out != NULL.  The first call for a
 * token count captures a CUDA graph (run it before any outer stream capture). */
int hpc_model_forward(hpc_model model, const int32_t *d_token_ids, const int32_t *d_positions, size_t token_count,
                      size_t top_k, int32_t *d_ids, float *d_vals, float *d_hidden_out, void *stream);

/* Prefill: token_count (1..context) hidden vectors [token_count][hidden]
 * (the embedding output, f32) at consecutive positions d_positions[0] + i
 * through every layer.  It writes every token's K/V into the cache and the
 * final residual stream to d_hidden_out [token_count][hidden].  This is the
 * reference's SegmentRunner.runTokensHidden / prefill path
 * (runner/segment-runner.ts:18-34, forward.ts:128-161;
 * runner/webgpu/segment-runner.ts:1292-1795 runBatchedPrefillFromBoundary).
 * Inputs of >= 16 columns run the matmuls on the tensor cores.  The
 * attention is causal over [0, position].  The launches are eager (no graph):
 * the call reads d_positions[0] back to size the attention's key windows (one
 * synchronization of `stream` per call), and the workspace grows to the
 * largest token count seen. */
int hpc_model_prefill(hpc_model model, const float *d_hidden_in, const int32_t *d_positions, size_t token_count,
                      float *d_hidden_out, void *stream);

/* ---- MTP draft head ("MTP assistant") -----------------------------------
 * runWasmMtpAssistant (runner/wasm/mtp-assistant-runner.ts:43-242) on the
 * GPU: pre projection over [target embedding ; target hidden], the draft
 * layers attending over the TARGET's KV cache, output norm, post projection
 * and maskedEmbeddingTopTokens (top centroids -> token ordering -> embedding
 * rows . h).  The matmuls are f32 products of the bit-exactly dequantized
 * weights (hp_matmul_dequantized_f32, lib.rs:103-154); each matrix is
 * dequantized once into the draft head's own f32 copy when it is set, so the
 * handles may be released afterwards.  One step is one CUDA graph. */

typedef struct hpc_draft_s *hpc_draft;

typedef struct {
  int backbone;       /* target hidden size */
  int hidden;         /* draft width (multiple of 256, <= 8192) */
  int heads;
  int kv_heads;       /* the target's KV heads */
  int head_dim;       /* 256 */
  int ffn;
  int vocab;
  int n_centroids;    /* <= 4096 */
  int centroid_top_k;
  int layers;
  int context;        /* largest position + 1 (multiple of 64, <= 4096) */
  int max_top_k;      /* 1..64 */
  double rms_eps;
  double rope_theta;
} hpc_draft_config;

/* matrices: per layer (layer index applies) */
#define HPC_DW_Q 0
#define HPC_DW_O 1
#define HPC_DW_GATE 2
#define HPC_DW_UP 3
#define HPC_DW_DOWN 4
#define HPC_DW_LAYER_COUNT 5
/* matrices: head-wide (layer ignored) */
#define HPC_DW_PRE 100       /* mtp.pre_projection.weight  [hidden][2 * backbone] */
#define HPC_DW_POST 101      /* mtp.post_projection.weight [backbone][hidden] */
#define HPC_DW_CENTROIDS 102 /* mtp.centroids.weight       [n_centroids][hidden] */
#define HPC_DW_EMBD 103      /* token_embd.weight          [vocab][hidden] */
/* f32 vectors */
#define HPC_DN_ATTN 0
#define HPC_DN_Q 1           /* attn_q_norm, head_dim values */
#define HPC_DN_POST_ATTN 2
#define HPC_DN_FFN 3
#define HPC_DN_POST_FFW 4
#define HPC_DN_LAYER_COUNT 5
#define HPC_DN_OUTPUT 100    /* output_norm (layer ignored) */

int hpc_draft_create(const hpc_draft_config *config, hpc_draft *out_draft);
int hpc_draft_release(hpc_draft draft);
int hpc_draft_set_matrix(hpc_draft draft, int which, int layer, hpc_weight weight);
int hpc_draft_set_vector(hpc_draft draft, int which, int layer, const float *host_values, size_t len);
int hpc_draft_set_layer_scale(hpc_draft draft, int layer, float scale);
/* token_ordering: n_centroids * per entries; centroid c lists its tokens at
 * [c * per, (c + 1) * per); centroid_top_k * per <= 4096 */
int hpc_draft_set_token_ordering(hpc_draft draft, const int32_t *host_ordering, size_t len);
/* The mapped target KV layer of draft layer `layer` (model.ts:457-478), both
 * [context][kv_heads][head_dim] f32 -- the layout hpc_model_kv returns. */
int hpc_draft_set_target_kv(hpc_draft draft, int layer, const float *d_key, const float *d_value);
/* One draft step at the target context's position (proposeMtpDraft keeps it
 * constant, mtp-generation.ts:92-137): backbone hidden [backbone] and the
 * top_k (token id, logit) pairs, value desc / id asc, into device buffers. */
int hpc_draft_step(hpc_draft draft, const float *d_embedding, const float *d_hidden, int position, size_t top_k,
                   float *d_post_out, int32_t *d_ids, float *d_vals, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* HELIOCUDA_H */
