// hc_model.cu -- resident decoder model and the decode / verify step.
//
// One call runs a whole forward pass for `token_count` consecutive tokens
// (decode: 1; MTP batched verify: 1 + drafts) and returns the top-k of every
// position.  It replaces the WASM provider's per-token graph
// (runner/wasm/layers.ts:161-473 forwardAttentionLayer + forwardFfn per layer,
// forwardOutput :381-416) and the WebGPU batched verify forward
// (runner/webgpu/segment-runner.ts:1292-1606 runBatchedPrefillFromBoundary,
// with per-position top-k :1441-1450).
//
// Kernel chain per layer (all launched with programmatic dependent launch):
//   [norm+quant] QKV GEMV (one launch) -> QK-norm/RoPE/KV write + split-KV
//   attention -> combine + f16 cast + quant -> O GEMV -> post-attention
//   residual + FFN norm + quant -> gate/up GEMV (one launch) -> GEGLU + quant
//   -> down GEMV -> post-FFN residual + next layer's attention norm + quant.
// The whole step is captured once per token count into a CUDA graph; inputs
// and outputs go through model-owned buffers so replays read current values.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/heliocuda.h"
#include "hc_common.cuh"
#include "hc_decode.cuh"
#include "hc_internal.h"
#include "hc_kernels.cuh"
#include "hc_lmhead.cuh"

namespace {

constexpr uint32_t kModelMagic = 0x48504d44u;  // "HPMD"

struct Layer {
  hpc_weight w[HPC_W_COUNT] = {};
  float* norm[HPC_N_COUNT] = {};  // device f32
};

}  // namespace

struct hpc_model_s {
  uint32_t magic = 0;
  int device = 0;
  hpc_model_config cfg{};
  std::vector<Layer> layers;
  float* output_norm = nullptr;
  hpc_weight lm_head = nullptr;
  std::vector<float*> kc, vc;  // per KV layer
  std::vector<int> kv_source;  // layer -> KV layer index
  // workspaces (sized for cfg.max_tokens columns)
  void* arena = nullptr;
  size_t arena_bytes = 0;
  float *x = nullptr, *h1 = nullptr, *qb = nullptr, *kb = nullptr, *vb = nullptr, *o = nullptr, *g = nullptr,
        *u = nullptr, *f = nullptr;
  float *pm = nullptr, *pl = nullptr, *po = nullptr;
  double *cos_t = nullptr, *sin_t = nullptr;
  int32_t *ids = nullptr, *pos = nullptr, *out_ids = nullptr;
  float* out_vals = nullptr;
  void* q8d = nullptr;  // Q8_K workspace for width D
  void* q8f = nullptr;  // Q8_K workspace for width F
  size_t q8d_bytes = 0, q8f_bytes = 0;
  void* cand = nullptr;
  size_t cand_bytes = 0;
  int* err = nullptr;
  // RoPE cos/sin of positions 0 .. rope_rows - 1 (twice the KV capacity, at
  // least 1024: decoding continues past the context on the slot ring),
  // computed once on the host (the C library's cos/sin) --
  // [rope_rows][head_dim / 2] each; later positions use the device's f64
  // cos/sin
  double *cos_tab = nullptr, *sin_tab = nullptr;
  int rope_rows = 0;
  // exact (default): every step in the reference's arithmetic order, its
  // results bit-identical to the WASM provider's; else the reordered kernels
  bool exact = true;
  float* attx_scratch = nullptr;  // exact attention: scores and probabilities
  float* attn16 = nullptr;        // exact attention: the f16-cast output [M][H * head_dim]
  std::mutex mu;
  // graph per token count
  std::vector<cudaGraphExec_t> graphs;
  std::vector<int> graph_k;
  cudaStream_t capture_stream = nullptr;
  // side stream of the step's L2 prefetches (forks after each QKV launch,
  // joins at the end of the step) and its fork / join events
  cudaStream_t side = nullptr;
  cudaEvent_t fork_ev = nullptr, join_ev = nullptr;
  bool l2_prefetch = false;
  // prefill workspace (hpc_model_prefill), grown to the largest token count seen
  void* pf_arena = nullptr;
  int pf_cap = 0;
  float *pf_x = nullptr, *pf_q = nullptr, *pf_k = nullptr, *pf_v = nullptr, *pf_qh = nullptr, *pf_o = nullptr,
        *pf_g = nullptr, *pf_u = nullptr, *pf_f = nullptr;
  double *pf_cos = nullptr, *pf_sin = nullptr;
  int32_t* pf_pos = nullptr;
  void *pf_q8d = nullptr, *pf_q8f = nullptr;
  void* pf_part = nullptr;  // split-attention partials (grows with tokens x splits)
  size_t pf_part_bytes = 0;
  size_t pf_q8d_bytes = 0, pf_q8f_bytes = 0;
};

static bool model_valid(const hpc_model_s* m) { return m && m->magic == kModelMagic; }

static int check_cfg(const hpc_model_config* c) {
  if (!c) return hpc_fail(HPC_ERR_ARG, "null config");
  if (c->hidden <= 0 || c->hidden % 2048 != 0 || c->hidden > 8192)
    return hpc_fail(HPC_ERR_SHAPE, "hidden size %d: must be a multiple of 2048 (<= 8192)", c->hidden);
  if (c->head_dim != 256) return hpc_fail(HPC_ERR_SHAPE, "head_dim %d: only 256 is supported", c->head_dim);
  if (c->heads <= 0 || c->kv_heads <= 0 || c->heads % c->kv_heads != 0 || c->heads * c->head_dim != c->hidden ||
      c->heads + 2 * c->kv_heads > 32)
    return hpc_fail(HPC_ERR_HEADS, "heads %d / kv_heads %d", c->heads, c->kv_heads);
  if (c->ffn <= 0 || c->ffn % 2048 != 0) return hpc_fail(HPC_ERR_SHAPE, "ffn %d: must be a multiple of 2048", c->ffn);
  if (c->layers <= 0 || c->kv_layers <= 0 || c->kv_layers > c->layers)
    return hpc_fail(HPC_ERR_SHAPE, "layers %d / kv_layers %d", c->layers, c->kv_layers);
  if (c->context <= 0 || c->context % 64 != 0 || c->context > 4096 || c->vocab <= 0)
    return hpc_fail(HPC_ERR_SHAPE, "context %d: a multiple of 64 up to 4096; vocab %d", c->context, c->vocab);
  if (c->max_tokens < 1 || c->max_tokens > 8) return hpc_fail(HPC_ERR_SHAPE, "max_tokens %d: 1..8", c->max_tokens);
  // an attention CTA stages the queries of every token for its KV head: the
  // widest step must fit the attention kernels' shared memory
  const size_t att_smem = hc::attn_smem_bytes(c->max_tokens, c->heads, c->kv_heads);
  if (att_smem > hc::ATT_MAX_SMEM)
    return hpc_fail(HPC_ERR_SHAPE,
                    "max_tokens %d x %d query heads per KV head needs %zu bytes of attention shared memory (max %zu)",
                    c->max_tokens, c->heads / c->kv_heads, att_smem, hc::ATT_MAX_SMEM);
  if (c->top_k < 1 || c->top_k > hc::TOPK_MAX) return hpc_fail(HPC_ERR_SHAPE, "top_k %d", c->top_k);
  return HPC_OK;
}

extern "C" {

int hpc_model_create(const hpc_model_config* cfg, hpc_model* out) {
  if (!out) return hpc_fail(HPC_ERR_ARG, "null out");
  *out = nullptr;
  int rc = check_cfg(cfg);
  if (rc != HPC_OK) return rc;
  auto* m = new hpc_model_s;
  m->cfg = *cfg;
  HPC_CK(cudaGetDevice(&m->device), "cudaGetDevice");
  const hpc_model_config& c = m->cfg;
  m->layers.resize(c.layers);
  // KV sharing (model.ts:368-388 kvSourceLayers): layers >= kv_layers reuse
  // the last KV layer (every layer is full attention here).
  m->kv_source.resize(c.layers);
  for (int l = 0; l < c.layers; ++l) m->kv_source[l] = l < c.kv_layers ? l : c.kv_layers - 1;
  const size_t kv_elems = size_t(c.context) * c.kv_heads * c.head_dim;
  m->kc.assign(c.kv_layers, nullptr);
  m->vc.assign(c.kv_layers, nullptr);
  for (int l = 0; l < c.kv_layers; ++l) {
    cudaError_t e = cudaMalloc(&m->kc[l], kv_elems * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&m->vc[l], kv_elems * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(m->kc[l], 0, kv_elems * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(m->vc[l], 0, kv_elems * sizeof(float));
    if (e != cudaSuccess) {
      m->magic = kModelMagic;
      hpc_model_release(m);
      return hpc_cuda_fail(e, "KV cache allocation");
    }
  }
  // workspace arena
  const int M = c.max_tokens, D = c.hidden, F = c.ffn, H = c.heads, KVH = c.kv_heads, HD = c.head_dim;
  const int G = H / KVH, NQ = M * G, chunks = (c.context + hc::ATT_CHUNK - 1) / hc::ATT_CHUNK;
  m->q8d_bytes = hc::q8buf_bytes(D, M);
  m->q8f_bytes = hc::q8buf_bytes(F, M);
  struct Piece {
    void** p;
    size_t bytes;
  };
  std::vector<Piece> pieces = {
      {(void**)&m->x, sizeof(float) * M * D},
      {(void**)&m->h1, sizeof(float) * M * D},
      {(void**)&m->qb, sizeof(float) * M * H * HD},
      {(void**)&m->kb, sizeof(float) * M * KVH * HD},
      {(void**)&m->vb, sizeof(float) * M * KVH * HD},
      {(void**)&m->o, sizeof(float) * M * D},
      {(void**)&m->g, sizeof(float) * M * F},
      {(void**)&m->u, sizeof(float) * M * F},
      {(void**)&m->f, sizeof(float) * M * D},
      {(void**)&m->pm, sizeof(float) * chunks * KVH * NQ},
      {(void**)&m->pl, sizeof(float) * chunks * KVH * NQ},
      {(void**)&m->po, sizeof(float) * chunks * KVH * NQ * HD},
      {(void**)&m->cos_t, sizeof(double) * M * HD / 2},
      {(void**)&m->sin_t, sizeof(double) * M * HD / 2},
      {(void**)&m->ids, sizeof(int32_t) * M},
      {(void**)&m->pos, sizeof(int32_t) * M},
      {(void**)&m->out_ids, sizeof(int32_t) * M * hc::TOPK_MAX},
      {(void**)&m->out_vals, sizeof(float) * M * hc::TOPK_MAX},
      {&m->q8d, m->q8d_bytes},
      {&m->q8f, m->q8f_bytes},
      {(void**)&m->attx_scratch, sizeof(float) * hc::attx_scratch_floats(M, H, c.context)},
      {(void**)&m->attn16, sizeof(float) * M * H * HD},
  };
  size_t total = 0;
  for (auto& p : pieces) total += (p.bytes + 255) / 256 * 256;
  if (cudaMalloc(&m->arena, total) != cudaSuccess) {
    m->magic = kModelMagic;
    hpc_model_release(m);
    return hpc_fail(HPC_ERR_CUDA, "workspace allocation of %zu bytes failed", total);
  }
  cudaMemset(m->arena, 0, total);
  m->arena_bytes = total;
  char* cur = static_cast<char*>(m->arena);
  for (auto& p : pieces) {
    *p.p = cur;
    cur += (p.bytes + 255) / 256 * 256;
  }
  m->err = hc::device_status_word();
  {
    // layers.ts:1012-1030: theta_0 = position, theta_{i+1} = fround(theta_i *
    // base^(-2/ndims)), cos/sin in f64 -- evaluated here with the host's
    // cos/sin, the same functions the reference's Math.cos/Math.sin and the
    // oracle use, so the angles' roundings do not depend on the device's
    // math library
    const int half = HD / 2;
    const double theta_scale = std::pow(c.rope_theta, -2.0 / double(HD));
    m->rope_rows = std::max(2 * c.context, 1024);
    std::vector<double> ct(size_t(m->rope_rows) * half), st(size_t(m->rope_rows) * half);
    for (int p = 0; p < m->rope_rows; ++p) {
      double th = double(p);
      for (int i = 0; i < half; ++i) {
        ct[size_t(p) * half + i] = std::cos(th);
        st[size_t(p) * half + i] = std::sin(th);
        th = double(float(th * theta_scale));
      }
    }
    cudaError_t e = cudaMalloc(&m->cos_tab, ct.size() * sizeof(double));
    if (e == cudaSuccess) e = cudaMalloc(&m->sin_tab, st.size() * sizeof(double));
    if (e == cudaSuccess) e = cudaMemcpy(m->cos_tab, ct.data(), ct.size() * sizeof(double), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(m->sin_tab, st.data(), st.size() * sizeof(double), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      m->magic = kModelMagic;
      hpc_model_release(m);
      return hpc_cuda_fail(e, "RoPE table");
    }
  }
  HPC_CK(cudaStreamCreateWithFlags(&m->capture_stream, cudaStreamNonBlocking), "cudaStreamCreate");
  HPC_CK(cudaStreamCreateWithFlags(&m->side, cudaStreamNonBlocking), "cudaStreamCreate");
  HPC_CK(cudaEventCreateWithFlags(&m->fork_ev, cudaEventDisableTiming), "cudaEventCreate");
  HPC_CK(cudaEventCreateWithFlags(&m->join_ev, cudaEventDisableTiming), "cudaEventCreate");
  {
    // HPC_DECODE_L2_PREFETCH=1 turns the per-layer weight prefetch on
    // (measured: it slowed the reordered step, 1.73 -> 2.35 ms)
    const char* e = getenv("HPC_DECODE_L2_PREFETCH");
    m->l2_prefetch = e && e[0] == '1';
  }
  m->graphs.assign(M + 1, nullptr);
  m->graph_k.assign(M + 1, 0);
  m->magic = kModelMagic;
  *out = m;
  return HPC_OK;
}

int hpc_model_release(hpc_model m) {
  if (!model_valid(m)) return hpc_fail(HPC_ERR_ARG, "invalid model");
  for (auto g : m->graphs)
    if (g) cudaGraphExecDestroy(g);
  for (auto p : m->kc) cudaFree(p);
  for (auto p : m->vc) cudaFree(p);
  for (auto& L : m->layers)
    for (auto n : L.norm) cudaFree(n);
  cudaFree(m->output_norm);
  cudaFree(m->cos_tab);
  cudaFree(m->sin_tab);
  cudaFree(m->arena);
  cudaFree(m->cand);
  cudaFree(m->pf_arena);
  cudaFree(m->pf_part);
  if (m->capture_stream) cudaStreamDestroy(m->capture_stream);
  if (m->side) cudaStreamDestroy(m->side);
  if (m->fork_ev) cudaEventDestroy(m->fork_ev);
  if (m->join_ev) cudaEventDestroy(m->join_ev);
  m->magic = 0;
  delete m;
  return HPC_OK;
}

static void invalidate_graphs(hpc_model m) {
  for (auto& g : m->graphs) {
    if (g) cudaGraphExecDestroy(g);
    g = nullptr;
  }
}

int hpc_model_set_weight(hpc_model m, int layer, int slot, hpc_weight w) {
  if (!model_valid(m)) return hpc_fail(HPC_ERR_ARG, "invalid model");
  if (layer < 0 || layer >= m->cfg.layers || slot < 0 || slot >= HPC_W_COUNT)
    return hpc_fail(HPC_ERR_ARG, "layer %d / slot %d", layer, slot);
  if (!hpc_weight_valid(w)) return hpc_fail(HPC_ERR_ARG, "invalid weight handle");
  const hpc_model_config& c = m->cfg;
  size_t K = c.hidden, N = 0;
  switch (slot) {
    case HPC_W_Q: N = size_t(c.heads) * c.head_dim; break;
    case HPC_W_K: case HPC_W_V: N = size_t(c.kv_heads) * c.head_dim; break;
    case HPC_W_O: K = size_t(c.heads) * c.head_dim; N = c.hidden; break;
    case HPC_W_GATE: case HPC_W_UP: N = c.ffn; break;
    case HPC_W_DOWN: K = c.ffn; N = c.hidden; break;
  }
  if ((slot == HPC_W_K || slot == HPC_W_V) && layer >= c.kv_layers)
    return hpc_fail(HPC_ERR_SHAPE, "layer %d shares KV and has no %s weight", layer, slot == HPC_W_K ? "K" : "V");
  if (w->input_size != K || w->row_count != N)
    return hpc_fail(HPC_ERR_SHAPE, "weight %zux%zu, expected %zux%zu", w->input_size, w->row_count, K, N);
  if (w->device != m->device) return hpc_fail(HPC_ERR_ARG, "weight on device %d, model on %d", w->device, m->device);
  m->layers[layer].w[slot] = w;
  invalidate_graphs(m);
  return HPC_OK;
}

int hpc_model_set_norm(hpc_model m, int layer, int slot, const float* host_values, size_t len) {
  if (!model_valid(m)) return hpc_fail(HPC_ERR_ARG, "invalid model");
  const hpc_model_config& c = m->cfg;
  float** dst;
  size_t want;
  if (slot == HPC_N_OUTPUT) {
    dst = &m->output_norm;
    want = c.hidden;
  } else {
    if (layer < 0 || layer >= c.layers || slot < 0 || slot >= HPC_N_COUNT)
      return hpc_fail(HPC_ERR_ARG, "layer %d / slot %d", layer, slot);
    dst = &m->layers[layer].norm[slot];
    want = (slot == HPC_N_Q || slot == HPC_N_K) ? size_t(c.head_dim) : size_t(c.hidden);
  }
  if (len != want || !host_values) return hpc_fail(HPC_ERR_SHAPE, "norm length %zu, expected %zu", len, want);
  if (!*dst) HPC_CK(cudaMalloc(dst, want * sizeof(float)), "cudaMalloc(norm)");
  HPC_CK(cudaMemcpy(*dst, host_values, want * sizeof(float), cudaMemcpyHostToDevice), "norm upload");
  return HPC_OK;
}

int hpc_model_set_lm_head(hpc_model m, hpc_weight w) {
  if (!model_valid(m)) return hpc_fail(HPC_ERR_ARG, "invalid model");
  if (!hpc_weight_valid(w)) return hpc_fail(HPC_ERR_ARG, "invalid weight handle");
  if (w->input_size != size_t(m->cfg.hidden) || w->row_count != size_t(m->cfg.vocab))
    return hpc_fail(HPC_ERR_SHAPE, "LM head %zux%zu", w->input_size, w->row_count);
  m->lm_head = w;
  // the candidate layout depends on the kernel a column count selects, so the
  // buffer serves the largest need over every token count of a step
  size_t cb = 0;
  for (int cols = 1; cols <= m->cfg.max_tokens; ++cols) {
    size_t need = 0;
    int rc = hpc_lm_head_candidates_bytes(w, size_t(cols), size_t(m->cfg.top_k), &need);
    if (rc != HPC_OK) return rc;
    if (need > cb) cb = need;
  }
  if (cb > m->cand_bytes) {
    cudaFree(m->cand);
    m->cand = nullptr;
    HPC_CK(cudaMalloc(&m->cand, cb), "cudaMalloc(candidates)");
    m->cand_bytes = cb;
  }
  invalidate_graphs(m);
  return HPC_OK;
}

int hpc_model_set_exact(hpc_model m, int enable) {
  if (!model_valid(m)) return hpc_fail(HPC_ERR_ARG, "invalid model");
  std::lock_guard<std::mutex> lock(m->mu);
  m->exact = enable != 0;
  invalidate_graphs(m);
  return HPC_OK;
}

int hpc_model_kv(hpc_model m, int kv_layer, float** d_key, float** d_value) {
  if (!model_valid(m)) return hpc_fail(HPC_ERR_ARG, "invalid model");
  if (kv_layer < 0 || kv_layer >= m->cfg.kv_layers) return hpc_fail(HPC_ERR_ARG, "kv layer %d", kv_layer);
  if (d_key) *d_key = m->kc[kv_layer];
  if (d_value) *d_value = m->vc[kv_layer];
  return HPC_OK;
}

}  // extern "C"

// Enqueues the whole step for M tokens on `st` (inputs already in m->ids/pos).
static int enqueue_step(hpc_model m, int M, int k, cudaStream_t st) {
  const hpc_model_config& c = m->cfg;
  const int D = c.hidden, F = c.ffn, H = c.heads, KVH = c.kv_heads, HD = c.head_dim;
  const double eps = c.rms_eps;
  const hc::Q8Buf qd = hc::q8buf_carve(m->q8d, D, M);
  const hc::Q8Buf qf = hc::q8buf_carve(m->q8f, F, M);
  auto mm = [&](std::initializer_list<std::pair<hpc_weight, float*>> ws, const void* q8, size_t q8_bytes,
                size_t K) -> int {
    hpc_weight hs[8];
    float* outs[8];
    size_t lens[8];
    int n = 0;
    for (auto& p : ws) {
      hs[n] = p.first;
      outs[n] = p.second;
      lens[n] = p.first->row_count * size_t(M);
      ++n;
    }
    return hc_matmul_q8_order(size_t(n), hs, q8, q8_bytes, K, size_t(M), outs, lens, m->exact, st);
  };
  const hpc_weight emb = m->lm_head;
  HPC_CK(hc::launch_rope_gather(m->pos, M, HD / 2, m->cos_tab, m->sin_tab, m->rope_rows,
                                std::pow(c.rope_theta, -2.0 / double(HD)), m->cos_t, m->sin_t, st),
         "rope rows");
  HPC_CK(hc::launch_embed(emb->d_data, emb->type, emb->nb, c.vocab, m->ids, m->x, M, D, std::sqrt(double(D)), m->err,
                          st),
         "embedding");
  // One or two columns of width 2048: the RMSNorms (+ residual adds) that feed
  // the QKV and gate/up projections are folded into those GEMVs (every CTA
  // computes them, hc_gemv.cu gemv_prologue).  The residual stream then
  // alternates between X (x_l, stored by the QKV prologue) and H1 (the
  // post-attention residual, stored by the gate/up prologue), so no CTA
  // overwrites a vector other CTAs of the same launch still read.
  // The exact step folds them the same way into its exact-order GEMVs, at
  // every width up to 8, and also the Q8_K of the attention output into the
  // O projection.
  const bool fused = (m->exact || M <= 2) && D == hc::GEMV_PRO_D;
  float* const X = m->x;
  float* const H1 = fused ? m->h1 : m->x;
  auto mm_pro = [&](std::initializer_list<std::pair<hpc_weight, float*>> ws, const hc::GemvPrologue& pro) -> int {
    hpc_weight hs[8];
    float* outs[8];
    size_t lens[8];
    int n = 0;
    for (auto& p : ws) {
      hs[n] = p.first;
      outs[n] = p.second;
      lens[n] = p.first->row_count * size_t(M);
      ++n;
    }
    if (m->exact)
      return hc_matmul_q8_exact_prologue(size_t(n), hs, m->q8d, m->q8d_bytes, size_t(D), size_t(M), outs, lens, pro,
                                         st);
    return hc_matmul_q8_prologue(size_t(n), hs, m->q8d, m->q8d_bytes, size_t(D), size_t(M), outs, lens, pro, st);
  };
  for (int l = 0; l < c.layers; ++l) {
    Layer& L = m->layers[l];
    const bool own_kv = l < c.kv_layers;
    const int kvl = m->kv_source[l];
    int rc;
    // attention norm (+ the previous layer's post-FFN residual) and QKV
    if (fused) {
      hc::GemvPrologue pro{};
      pro.eps = eps;
      pro.w_pre = L.norm[HPC_N_ATTN];
      if (l == 0) {
        pro.mode = hc::GEMV_PRO_NORM;
        pro.x = X;
      } else {
        pro.mode = hc::GEMV_PRO_RESID_NORM;
        pro.x = H1;
        pro.y = m->f;
        pro.w_post = m->layers[l - 1].norm[HPC_N_POST_FFW];
        pro.x_out = X;
      }
      rc = own_kv ? mm_pro({{L.w[HPC_W_Q], m->qb}, {L.w[HPC_W_K], m->kb}, {L.w[HPC_W_V], m->vb}}, pro)
                  : mm_pro({{L.w[HPC_W_Q], m->qb}}, pro);
    } else {
      if (l == 0) {
        HPC_CK(hc::launch_norm_quant(false, X, X, nullptr, nullptr, L.norm[HPC_N_ATTN], eps, M, D, qd, nullptr, st),
               "attn norm");
      } else {
        HPC_CK(hc::launch_norm_quant(true, X, X, m->f, m->layers[l - 1].norm[HPC_N_POST_FFW], L.norm[HPC_N_ATTN], eps,
                                     M, D, qd, nullptr, st),
               "post-ffn residual + attn norm");
      }
      rc = own_kv ? mm({{L.w[HPC_W_Q], m->qb}, {L.w[HPC_W_K], m->kb}, {L.w[HPC_W_V], m->vb}}, m->q8d, m->q8d_bytes, D)
                  : mm({{L.w[HPC_W_Q], m->qb}}, m->q8d, m->q8d_bytes, D);
    }
    if (rc != HPC_OK) return rc;
    if (m->l2_prefetch) {
      // while the attention runs: this layer's O, gate, up and down weights into L2
      hc::PrefetchList pl{};
      for (int slot : {HPC_W_O, HPC_W_GATE, HPC_W_UP, HPC_W_DOWN}) {
        pl.ptr[pl.n] = L.w[slot]->d_data;
        pl.bytes[pl.n] = L.w[slot]->bytes;
        ++pl.n;
      }
      HPC_CK(cudaEventRecord(m->fork_ev, st), "fork record");
      HPC_CK(cudaStreamWaitEvent(m->side, m->fork_ev, 0), "fork wait");
      HPC_CK(hc::launch_l2_prefetch(pl, m->side), "L2 prefetch");
    }
    if (m->exact) {
      HPC_CK(hc::launch_attention_exact(m->qb, m->kb, m->vb, L.norm[HPC_N_Q], L.norm[HPC_N_K], m->cos_t, m->sin_t, eps,
                                        own_kv, m->kc[kvl], m->vc[kvl], m->pos, M, H, KVH, c.context, 1.0f,
                                        m->attx_scratch, m->attn16, st),
             "exact-order attention");
    } else {
      HPC_CK(hc::launch_attention(m->qb, m->kb, m->vb, L.norm[HPC_N_Q], L.norm[HPC_N_K], m->cos_t, m->sin_t, eps,
                                  own_kv, m->kc[kvl], m->vc[kvl], m->pos, M, H, KVH, c.context, 1.0f, m->pm, m->pl,
                                  m->po, m->err, st),
             "qk norm / rope / kv + attention");
      HPC_CK(hc::launch_attn_combine(m->pm, m->pl, m->po, m->pos, M, H, KVH, c.context, qd, nullptr, st),
             "attention combine");
    }
    if (m->exact && H * HD == hc::GEMV_PRO_D) {
      hc::GemvPrologue pro{};  // the O projection quantizes the f16-cast attention output itself
      pro.mode = hc::GEMV_PRO_QUANT;
      pro.x = m->attn16;
      rc = mm_pro({{L.w[HPC_W_O], m->o}}, pro);
    } else {
      if (m->exact)
        HPC_CK(hc::launch_q8k_quantize(m->attn16, H * HD, M, qd, nullptr, nullptr, nullptr, st), "attention quantize");
      rc = mm({{L.w[HPC_W_O], m->o}}, m->q8d, m->q8d_bytes, size_t(H) * HD);
    }
    if (rc != HPC_OK) return rc;
    // post-attention residual + FFN norm and gate/up
    if (fused) {
      hc::GemvPrologue pro{};
      pro.mode = hc::GEMV_PRO_RESID_NORM;
      pro.eps = eps;
      pro.x = X;
      pro.y = m->o;
      pro.w_post = L.norm[HPC_N_POST_ATTN];
      pro.w_pre = L.norm[HPC_N_FFN];
      pro.x_out = H1;
      rc = mm_pro({{L.w[HPC_W_GATE], m->g}, {L.w[HPC_W_UP], m->u}}, pro);
    } else {
      HPC_CK(hc::launch_norm_quant(true, X, X, m->o, L.norm[HPC_N_POST_ATTN], L.norm[HPC_N_FFN], eps, M, D, qd,
                                   nullptr, st),
             "post-attn residual + ffn norm");
      rc = mm({{L.w[HPC_W_GATE], m->g}, {L.w[HPC_W_UP], m->u}}, m->q8d, m->q8d_bytes, D);
    }
    if (rc != HPC_OK) return rc;
    HPC_CK(hc::launch_geglu_quant(m->g, m->u, M, F, qf, nullptr, st), "geglu");
    rc = mm({{L.w[HPC_W_DOWN], m->f}}, m->q8f, m->q8f_bytes, F);
    if (rc != HPC_OK) return rc;
  }
  if (m->l2_prefetch) {  // the side stream joins the step
    HPC_CK(cudaEventRecord(m->join_ev, m->side), "join record");
    HPC_CK(cudaStreamWaitEvent(st, m->join_ev, 0), "join wait");
  }
  // final post-FFN residual + output norm, then the LM head
  HPC_CK(hc::launch_norm_quant(true, H1, X, m->f, m->layers[c.layers - 1].norm[HPC_N_POST_FFW], m->output_norm, eps,
                               M, D, qd, nullptr, st),
         "post-ffn residual + output norm");
  return hc_lm_head_topk_q8_order(emb, m->q8d, m->q8d_bytes, size_t(D), size_t(M), size_t(k), 0, m->cand,
                                  m->cand_bytes, c.final_logit_softcap, m->out_ids, m->out_vals, nullptr, m->exact, st);
}

static int model_ready(hpc_model m) {
  const hpc_model_config& c = m->cfg;
  if (!m->lm_head || !m->output_norm) return hpc_fail(HPC_ERR_ARG, "LM head / output norm not set");
  for (int l = 0; l < c.layers; ++l) {
    const Layer& L = m->layers[l];
    for (int s = 0; s < HPC_W_COUNT; ++s) {
      if ((s == HPC_W_K || s == HPC_W_V) && l >= c.kv_layers) continue;
      if (!L.w[s]) return hpc_fail(HPC_ERR_ARG, "layer %d weight %d not set", l, s);
    }
    for (int s = 0; s < HPC_N_COUNT; ++s)
      if (!L.norm[s]) return hpc_fail(HPC_ERR_ARG, "layer %d norm %d not set", l, s);
  }
  return HPC_OK;
}

extern "C" {

int hpc_model_forward(hpc_model m, const int32_t* d_token_ids, const int32_t* d_positions, size_t token_count,
                      size_t top_k, int32_t* d_ids, float* d_vals, float* d_hidden_out, void* stream) {
  if (!model_valid(m)) return hpc_fail(HPC_ERR_ARG, "invalid model");
  const hpc_model_config& c = m->cfg;
  if (token_count < 1 || token_count > size_t(c.max_tokens))
    return hpc_fail(HPC_ERR_SHAPE, "token count %zu outside 1..%d", token_count, c.max_tokens);
  if (top_k < 1 || top_k > size_t(c.top_k)) return hpc_fail(HPC_ERR_SHAPE, "top_k %zu outside 1..%d", top_k, c.top_k);
  if (!d_token_ids || !d_positions || !d_ids || !d_vals) return hpc_fail(HPC_ERR_ARG, "null pointer");
  int rc = model_ready(m);
  if (rc != HPC_OK) return rc;
  int dev = 0;
  HPC_CK(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != m->device) return hpc_fail(HPC_ERR_ARG, "model on device %d, current %d", m->device, dev);
  std::lock_guard<std::mutex> lock(m->mu);
  const int M = int(token_count), k = int(top_k);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  HPC_CK(cudaMemcpyAsync(m->ids, d_token_ids, sizeof(int32_t) * M, cudaMemcpyDeviceToDevice, st), "ids copy");
  HPC_CK(cudaMemcpyAsync(m->pos, d_positions, sizeof(int32_t) * M, cudaMemcpyDeviceToDevice, st), "positions copy");
  if (!m->graphs[M] || m->graph_k[M] != k) {
    if (m->graphs[M]) cudaGraphExecDestroy(m->graphs[M]);
    m->graphs[M] = nullptr;
    // Warm-up run outside capture (sets kernel attributes, validates), then capture.
    rc = enqueue_step(m, M, k, st);
    if (rc != HPC_OK) return rc;
    cudaStream_t cs = m->capture_stream;
    cudaEvent_t ev;
    HPC_CK(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "event");
    cudaEventRecord(ev, st);
    cudaStreamWaitEvent(cs, ev, 0);
    cudaEventDestroy(ev);
    HPC_CK(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal), "begin capture");
    rc = enqueue_step(m, M, k, cs);
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(cs, &graph);
    if (rc != HPC_OK) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    if (e != cudaSuccess) return hpc_cuda_fail(e, "end capture");
    e = cudaGraphInstantiate(&m->graphs[M], graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return hpc_cuda_fail(e, "graph instantiate");
    m->graph_k[M] = k;
    cudaEvent_t ev2;
    cudaEventCreateWithFlags(&ev2, cudaEventDisableTiming);
    cudaEventRecord(ev2, cs);
    cudaStreamWaitEvent(st, ev2, 0);
    cudaEventDestroy(ev2);
  } else {
    HPC_CK(cudaGraphLaunch(m->graphs[M], st), "graph launch");
  }
  HPC_CK(cudaMemcpyAsync(d_ids, m->out_ids, sizeof(int32_t) * M * k, cudaMemcpyDeviceToDevice, st), "ids out");
  HPC_CK(cudaMemcpyAsync(d_vals, m->out_vals, sizeof(float) * M * k, cudaMemcpyDeviceToDevice, st), "vals out");
  if (d_hidden_out)
    HPC_CK(cudaMemcpyAsync(d_hidden_out, m->x, sizeof(float) * M * c.hidden, cudaMemcpyDeviceToDevice, st),
           "hidden out");
  return HPC_OK;
}


}  // extern "C"

// Grows the prefill workspace to `M` tokens (one arena; the old one is freed).
static int prefill_reserve(hpc_model m, int M) {
  if (M <= m->pf_cap) return HPC_OK;
  const hpc_model_config& c = m->cfg;
  const int D = c.hidden, F = c.ffn, H = c.heads, KVH = c.kv_heads, HD = c.head_dim;
  cudaFree(m->pf_arena);
  m->pf_arena = nullptr;
  m->pf_cap = 0;
  m->pf_q8d_bytes = hc::q8buf_bytes(D, M);
  m->pf_q8f_bytes = hc::q8buf_bytes(F, M);
  struct Piece {
    void** p;
    size_t bytes;
  };
  std::vector<Piece> pieces = {
      {(void**)&m->pf_x, sizeof(float) * M * D},          {(void**)&m->pf_q, sizeof(float) * M * H * HD},
      {(void**)&m->pf_k, sizeof(float) * M * KVH * HD},   {(void**)&m->pf_v, sizeof(float) * M * KVH * HD},
      {(void**)&m->pf_qh, sizeof(float) * M * H * HD},    {(void**)&m->pf_o, sizeof(float) * M * D},
      {(void**)&m->pf_g, sizeof(float) * M * F},          {(void**)&m->pf_u, sizeof(float) * M * F},
      {(void**)&m->pf_f, sizeof(float) * M * D},          {(void**)&m->pf_cos, sizeof(double) * M * HD / 2},
      {(void**)&m->pf_sin, sizeof(double) * M * HD / 2},  {(void**)&m->pf_pos, sizeof(int32_t) * M},
      {&m->pf_q8d, m->pf_q8d_bytes},                      {&m->pf_q8f, m->pf_q8f_bytes},
  };
  size_t total = 0;
  for (auto& p : pieces) total += (p.bytes + 255) / 256 * 256;
  HPC_CK(cudaMalloc(&m->pf_arena, total), "prefill workspace");
  char* cur = static_cast<char*>(m->pf_arena);
  for (auto& p : pieces) {
    *p.p = cur;
    cur += (p.bytes + 255) / 256 * 256;
  }
  m->pf_cap = M;
  return HPC_OK;
}

extern "C" {

int hpc_model_prefill(hpc_model m, const float* d_hidden_in, const int32_t* d_positions, size_t token_count,
                      float* d_hidden_out, void* stream) {
  if (!model_valid(m)) return hpc_fail(HPC_ERR_ARG, "invalid model");
  const hpc_model_config& c = m->cfg;
  if (token_count < 1 || token_count > size_t(c.context))
    return hpc_fail(HPC_ERR_SHAPE, "prefill token count %zu outside 1..%d", token_count, c.context);
  if (!d_hidden_in || !d_positions || !d_hidden_out) return hpc_fail(HPC_ERR_ARG, "null pointer");
  int rc = model_ready(m);
  if (rc != HPC_OK) return rc;
  std::lock_guard<std::mutex> lock(m->mu);
  const int M = int(token_count);
  rc = prefill_reserve(m, M);
  if (rc != HPC_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int D = c.hidden, F = c.ffn, H = c.heads, KVH = c.kv_heads, HD = c.head_dim;
  const double eps = c.rms_eps;
  const hc::Q8Buf qd = hc::q8buf_carve(m->pf_q8d, D, M);
  const hc::Q8Buf qf = hc::q8buf_carve(m->pf_q8f, F, M);
  float* X = m->pf_x;
  HPC_CK(cudaMemcpyAsync(X, d_hidden_in, sizeof(float) * M * D, cudaMemcpyDeviceToDevice, st), "hidden in");
  HPC_CK(cudaMemcpyAsync(m->pf_pos, d_positions, sizeof(int32_t) * M, cudaMemcpyDeviceToDevice, st), "positions");
  // the split attention sizes its grid from the key window: the positions
  // are consecutive, so the first one bounds it (one small read per call)
  const int G = H / KVH;
  int nsplit = 0;
  float *pm = nullptr, *pl = nullptr, *po = nullptr;
  if (G <= 4) {
    int32_t pos0 = 0;
    HPC_CK(cudaMemcpyAsync(&pos0, d_positions, sizeof pos0, cudaMemcpyDeviceToHost, st), "first position");
    HPC_CK(cudaStreamSynchronize(st), "first position");
    if (pos0 < 0) return hpc_fail(HPC_ERR_SHAPE, "prefill position %d", pos0);
    nsplit = hc::prefill_attn_splits(c.context, pos0 + M - 1);
    const size_t rows = size_t(M) * H * nsplit;
    const size_t need = (rows * 2 * sizeof(float) + 255) / 256 * 256 + rows * HD * sizeof(float);
    if (need > m->pf_part_bytes) {
      cudaFree(m->pf_part);
      m->pf_part = nullptr;
      m->pf_part_bytes = 0;
      HPC_CK(cudaMalloc(&m->pf_part, need), "prefill attention partials");
      m->pf_part_bytes = need;
    }
    pm = static_cast<float*>(m->pf_part);
    pl = pm + rows;
    po = reinterpret_cast<float*>(static_cast<char*>(m->pf_part) + (rows * 2 * sizeof(float) + 255) / 256 * 256);
  }
  HPC_CK(hc::launch_rope_gather(m->pf_pos, M, HD / 2, m->cos_tab, m->sin_tab, m->rope_rows,
                                std::pow(c.rope_theta, -2.0 / double(HD)), m->pf_cos, m->pf_sin, st),
         "rope rows");
  auto mm = [&](std::initializer_list<std::pair<hpc_weight, float*>> ws, const void* q8, size_t q8_bytes,
                size_t K) -> int {
    hpc_weight hs[8];
    float* outs[8];
    size_t lens[8];
    int n = 0;
    for (auto& p : ws) {
      hs[n] = p.first;
      outs[n] = p.second;
      lens[n] = p.first->row_count * size_t(M);
      ++n;
    }
    return hpc_matmul_q8(size_t(n), hs, q8, q8_bytes, K, size_t(M), outs, lens, st);
  };
  for (int l = 0; l < c.layers; ++l) {
    Layer& L = m->layers[l];
    const bool own_kv = l < c.kv_layers;
    const int kvl = m->kv_source[l];
    if (l == 0)
      HPC_CK(hc::launch_norm_quant(false, X, X, nullptr, nullptr, L.norm[HPC_N_ATTN], eps, M, D, qd, nullptr, st),
             "attn norm");
    else
      HPC_CK(hc::launch_norm_quant(true, X, X, m->pf_f, m->layers[l - 1].norm[HPC_N_POST_FFW], L.norm[HPC_N_ATTN], eps,
                                   M, D, qd, nullptr, st),
             "post-ffn residual + attn norm");
    rc = own_kv ? mm({{L.w[HPC_W_Q], m->pf_q}, {L.w[HPC_W_K], m->pf_k}, {L.w[HPC_W_V], m->pf_v}}, m->pf_q8d,
                     m->pf_q8d_bytes, D)
                : mm({{L.w[HPC_W_Q], m->pf_q}}, m->pf_q8d, m->pf_q8d_bytes, D);
    if (rc != HPC_OK) return rc;
    HPC_CK(hc::launch_prefill_qkv_post(m->pf_q, m->pf_k, m->pf_v, L.norm[HPC_N_Q], L.norm[HPC_N_K], m->pf_cos,
                                       m->pf_sin, eps, own_kv, m->kc[kvl], m->vc[kvl], m->pf_pos, M, H, KVH, c.context,
                                       m->pf_qh, st),
           "prefill qk norm / rope / kv");
    if (nsplit > 0)
      HPC_CK(hc::launch_prefill_attention_split(m->pf_qh, m->kc[kvl], m->vc[kvl], m->pf_pos, M, H, KVH, c.context,
                                                nsplit, pm, pl, po, qd, nullptr, st),
             "prefill attention");
    else
      HPC_CK(hc::launch_prefill_attention(m->pf_qh, m->kc[kvl], m->vc[kvl], m->pf_pos, M, H, KVH, c.context, qd, nullptr,
                                        st),
           "prefill attention");
    rc = mm({{L.w[HPC_W_O], m->pf_o}}, m->pf_q8d, m->pf_q8d_bytes, size_t(H) * HD);
    if (rc != HPC_OK) return rc;
    HPC_CK(hc::launch_norm_quant(true, X, X, m->pf_o, L.norm[HPC_N_POST_ATTN], L.norm[HPC_N_FFN], eps, M, D, qd,
                                 nullptr, st),
           "post-attn residual + ffn norm");
    rc = mm({{L.w[HPC_W_GATE], m->pf_g}, {L.w[HPC_W_UP], m->pf_u}}, m->pf_q8d, m->pf_q8d_bytes, D);
    if (rc != HPC_OK) return rc;
    HPC_CK(hc::launch_geglu_quant(m->pf_g, m->pf_u, M, F, qf, nullptr, st), "geglu");
    rc = mm({{L.w[HPC_W_DOWN], m->pf_f}}, m->pf_q8f, m->pf_q8f_bytes, F);
    if (rc != HPC_OK) return rc;
  }
  // the last post-FFN residual (the output norm's quantization is computed
  // and discarded: prefill returns the residual stream)
  HPC_CK(hc::launch_norm_quant(true, X, X, m->pf_f, m->layers[c.layers - 1].norm[HPC_N_POST_FFW], m->output_norm, eps,
                               M, D, qd, nullptr, st),
         "post-ffn residual");
  HPC_CK(cudaMemcpyAsync(d_hidden_out, X, sizeof(float) * M * D, cudaMemcpyDeviceToDevice, st), "hidden out");
  return HPC_OK;
}

}  // extern "C"
