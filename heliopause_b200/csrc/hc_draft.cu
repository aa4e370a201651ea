// hc_draft.cu -- the MTP draft head ("MTP assistant") on the GPU.
//
// Restates runWasmMtpAssistant (packages/engine/src/runner/wasm/
// mtp-assistant-runner.ts:43-242) for one draft step:
//   x   = pre_projection @ [target embedding ; target hidden]            :43-66
//   per layer (attention over the TARGET's KV cache)                    :68-140
//     a = rmsNorm(x, attn_norm); q = normHeads(Wq a, q_norm); partial NeoX RoPE
//     o = Wo gqa_attention(q, K, V, causal to the position, scale 1, f32 query)
//     r = x + rmsNorm(o, post_attention_norm);  n = rmsNorm(r, ffn_norm)
//     f = r + rmsNorm(Wd fround(gelu(Wg n) * (Wu n)), post_ffw_norm)    :142-158
//     x = fround(f * layer_output_scale)
//   h   = rmsNorm(x, output_norm); post = post_projection @ h
//   top tokens = maskedEmbeddingTopTokens(h, centroids @ h)             :211-242
// The matmuls are matMulAssistantWeight (:160-183 -> hp_matmul_dequantized_f32,
// lib.rs:103-154): each weight element dequantized bit-exactly from the
// resident row tiles (the head keeps its own copy of the quantized bytes,
// 7x fewer than f32 rows) and one sequential f32 chain per output row in
// index order -- the reference's own sum, bit for bit
// (hc_dequant_matmul_kernel).  The masked token scores (:211-242) are the
// same chain over the gathered embedding rows.  Elsewhere rounding points
// follow the reference (f32 sums of squares and f64 norm scales, the f32
// theta chain of the partial RoPE with f64 cos/sin, f64 exp of f32 score
// differences, fround of the gated GELU) while the norm and attention sums
// run in parallel orders, so those agree to f32 rounding.
//
// One step is one CUDA graph (captured on first use, re-captured when the
// target KV pointers change): the position and top-k travel in device
// memory, written with the inputs by one small launch before the graph.
#include <cmath>
#include <cstring>
#include <vector>

#include "../../include/heliocuda.h"
#include "hc_bulk.cuh"
#include "hc_common.cuh"
#include "hc_decmath.cuh"
#include "hc_internal.h"
#include "hc_kernels.cuh"
#include "hc_unpack.cuh"

namespace hc {
namespace {

constexpr int DN_THREADS = 1024; // norm kernels: one CTA
constexpr int DA_CHUNK = 64;     // attention tokens per CTA
constexpr int DT_THREADS = 1024; // top-k selection: one CTA
constexpr int DT_MAXN = 4096;    // keys one selection sorts

// f32 sum of squares of v[0..n) over the CTA (every thread gets the total).
__device__ float block_sumsq_f32(const float* v, int n, float* red) {
  float s = 0.0f;
  for (int i = int(threadIdx.x); i < n; i += int(blockDim.x)) s = fmaf(v[i], v[i], s);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31), nw = int(blockDim.x >> 5);
  __syncthreads();
  if (lane == 0) red[warp] = s;
  __syncthreads();
  float t = 0.0f;
  for (int w = 0; w < nw; ++w) t += red[w];
  return t;
}

// rmsNorm (mtp-assistant-runner.ts:275-290): f32 sum of squares, f64 scale,
// fround(fround(x * scale) * w).
__device__ __forceinline__ float norm_elem(float x, double scale, float w) {
  return float(double(float(double(x) * scale)) * double(w));
}

// mode 0: out1 = rmsNorm(x, w1)
// mode 1: out1 = r = x + rmsNorm(y, w1); out2 = rmsNorm(r, w2)
// mode 2: out1 = fround((x + rmsNorm(y, w1)) * scale)
__global__ void __launch_bounds__(DN_THREADS) hc_dnorm_kernel(int mode, int n, const float* __restrict__ x,
                                                           const float* __restrict__ y, const float* __restrict__ w1,
                                                           const float* __restrict__ w2, double eps, float scale,
                                                           float* __restrict__ out1, float* __restrict__ out2) {
  __shared__ float red[32];
  extern __shared__ float buf[];  // n floats
  const float* src = mode == 0 ? x : y;
  const double sc = 1.0 / sqrt(double(block_sumsq_f32(src, n, red)) / double(n) + eps);
  if (mode == 0) {
    for (int i = int(threadIdx.x); i < n; i += int(blockDim.x)) out1[i] = norm_elem(x[i], sc, w1[i]);
    return;
  }
  for (int i = int(threadIdx.x); i < n; i += int(blockDim.x)) {
    const float r = x[i] + norm_elem(y[i], sc, w1[i]);
    if (mode == 2) {
      out1[i] = float(double(r) * double(scale));
    } else {
      out1[i] = r;
      buf[i] = r;
    }
  }
  if (mode != 1) return;
  __syncthreads();
  const double sc2 = 1.0 / sqrt(double(block_sumsq_f32(buf, n, red)) / double(n) + eps);
  for (int i = int(threadIdx.x); i < n; i += int(blockDim.x)) out2[i] = norm_elem(buf[i], sc2, w2[i]);
}

// normHeads with the q norm weight, then ropeNeox with activePairCount
// (mtp-assistant-runner.ts:361-387): only the first `pairs` pairs (i, i + hd/2)
// rotate; theta starts at the position and advances as
// fround(theta * base^(-2/hd)); cos/sin in f64.  One CTA per head, thread =
// dimension.
__global__ void __launch_bounds__(256) hc_dqrope_kernel(float* __restrict__ q, const float* __restrict__ qnw, int hd,
                                                     const int* __restrict__ pos, int pairs, double theta_scale,
                                                     double eps) {
  __shared__ float red[32];
  __shared__ float v[256];
  float* qh = q + size_t(blockIdx.x) * hd;
  const double sc = 1.0 / sqrt(double(block_sumsq_f32(qh, hd, red)) / double(hd) + eps);
  const int d = int(threadIdx.x);
  if (d < hd) v[d] = norm_elem(qh[d], sc, qnw[d]);
  __syncthreads();
  const int half = hd / 2;
  if (d < pairs) {
    double theta = double(*pos);
    for (int i = 0; i < d; ++i) theta = double(float(theta * theta_scale));
    const double x0 = v[d], x1 = v[half + d];
    const double c = cos(theta), s = sin(theta);
    qh[d] = float(x0 * c) - float(x1 * s);
    qh[half + d] = float(x0 * s) + float(x1 * c);
  } else if (d < half || (d >= half + pairs && d < hd)) {
    qh[d] = v[d];
  }
}

// GQA attention of one token's query heads over the target KV (K and V both
// [cap][kvh][hd], causal to *pos, scale 1, f32 query; lib.rs:539-654 as the
// draft head calls it): split over DA_CHUNK-token slices, local max / sum of
// f64 exp / sum of p * v per slice, merged by hc_dattn_combine_kernel.
// Grid (cap / DA_CHUNK, kvh); the slice's K and V rows are staged in shared
// memory first (all 16-byte copies in flight at once); thread d = dimension.
constexpr int DA_KSTRIDE = 256 + 4;  // floats per staged row (16-byte reads by consecutive tokens hit distinct banks)
__host__ __device__ constexpr size_t dattn_smem_floats(int G) {
  return size_t(G) * (256 + DA_CHUNK) + 2 * size_t(DA_CHUNK) * DA_KSTRIDE;
}
__global__ void __launch_bounds__(256) hc_dattn_partial_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                                            const float* __restrict__ vc, const int* __restrict__ pos,
                                                            int H, int KVH, float* __restrict__ part_m,
                                                            float* __restrict__ part_l, float* __restrict__ part_o) {
  constexpr int HD = 256, CH = DA_CHUNK;
  extern __shared__ __align__(16) float sm[];
  const int G = H / KVH, chunk = int(blockIdx.x), kvh = int(blockIdx.y);
  const int count = *pos + 1, t0 = chunk * CH;
  if (t0 >= count) return;
  const int nt = min(CH, count - t0);
  float* qs = sm;            // [G][HD]
  float* ps = qs + G * HD;   // [G][CH]
  float* ks = ps + G * CH;   // [CH][DA_KSTRIDE]
  float* vs = ks + CH * DA_KSTRIDE;
  for (int i = int(threadIdx.x); i < nt * (HD / 4); i += int(blockDim.x)) {
    const int t = i / (HD / 4), c4 = i % (HD / 4);
    const size_t src = (size_t(t0 + t) * KVH + kvh) * HD + 4 * c4;
    cp_async16(ks + t * DA_KSTRIDE + 4 * c4, kc + src);
    cp_async16(vs + t * DA_KSTRIDE + 4 * c4, vc + src);
  }
  cp_async_commit();
  for (int i = int(threadIdx.x); i < G * HD; i += int(blockDim.x)) qs[i] = q[size_t(kvh) * G * HD + i];
  cp_async_wait_all();
  __syncthreads();
  for (int pr = int(threadIdx.x); pr < G * CH; pr += int(blockDim.x)) {
    const int g = pr / CH, t = pr % CH;
    float dot = -INFINITY;
    if (t < nt) {
      const float4* kv = reinterpret_cast<const float4*>(ks + t * DA_KSTRIDE);
      const float4* qv = reinterpret_cast<const float4*>(qs + g * HD);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
      for (int j = 0; j < HD / 4; ++j) {
        const float4 a = qv[j], b = kv[j];
        acc.x = fmaf(a.x, b.x, acc.x);
        acc.y = fmaf(a.y, b.y, acc.y);
        acc.z = fmaf(a.z, b.z, acc.z);
        acc.w = fmaf(a.w, b.w, acc.w);
      }
      dot = (acc.x + acc.y) + (acc.z + acc.w);
    }
    ps[pr] = dot;
  }
  __syncthreads();
  const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31), warps = int(blockDim.x >> 5);
  for (int g = warp; g < G; g += warps) {
    float mx = -INFINITY;
    for (int t = lane; t < CH; t += 32) mx = fmaxf(mx, ps[g * CH + t]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.0f;
    for (int t = lane; t < CH; t += 32) {
      const float s = ps[g * CH + t];
      const float p = s == -INFINITY ? 0.0f : float(exp(double(s - mx)));
      ps[g * CH + t] = p;
      sum += p;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == 0) {
      part_m[(size_t(chunk) * KVH + kvh) * G + g] = mx;
      part_l[(size_t(chunk) * KVH + kvh) * G + g] = sum;
    }
  }
  __syncthreads();
  const int d = int(threadIdx.x);
  for (int g = 0; g < G; ++g) {
    float acc = 0.0f;
    for (int t = 0; t < nt; ++t) acc = fmaf(ps[g * CH + t], vs[t * DA_KSTRIDE + d], acc);
    part_o[((size_t(chunk) * KVH + kvh) * G + g) * HD + d] = acc;
  }
}

// Merges the slices of one head: global max, f64-exp slice weights, f64 sum,
// weighted outputs, division.  Grid H; thread d = dimension.
__global__ void __launch_bounds__(256) hc_dattn_combine_kernel(const float* __restrict__ part_m,
                                                            const float* __restrict__ part_l,
                                                            const float* __restrict__ part_o,
                                                            const int* __restrict__ pos, int H, int KVH,
                                                            float* __restrict__ out) {
  constexpr int HD = 256;
  __shared__ float w[4096 / DA_CHUNK];
  __shared__ double lsum;
  const int G = H / KVH, h = int(blockIdx.x), kvh = h / G, g = h % G, d = int(threadIdx.x);
  const int nch = (*pos + 1 + DA_CHUNK - 1) / DA_CHUNK;
  if (d == 0) {
    float mx = -INFINITY;
    for (int c = 0; c < nch; ++c) mx = fmaxf(mx, part_m[(size_t(c) * KVH + kvh) * G + g]);
    double l = 0.0;
    for (int c = 0; c < nch; ++c) {
      const float mc = part_m[(size_t(c) * KVH + kvh) * G + g];
      const float wc = mc == -INFINITY ? 0.0f : float(exp(double(mc - mx)));
      w[c] = wc;
      l += double(wc) * double(part_l[(size_t(c) * KVH + kvh) * G + g]);
    }
    lsum = l;
  }
  __syncthreads();
  float o = 0.0f;
  for (int c = 0; c < nch; ++c) o = fmaf(w[c], part_o[((size_t(c) * KVH + kvh) * G + g) * HD + d], o);
  out[size_t(h) * HD + d] = float(double(o) / lsum);
}

// gelu (mtp-assistant-runner.ts:399-411): tanh form with f32 rounding points,
// no f16 round trips; the gated product fround(gelu(gate) * up) (:150-153).
__device__ __forceinline__ double gelu_f32points(float v) {
  const double x = v;
  if (x <= -10.0) return 0.0;
  if (x >= 10.0) return x;
  const float a = float(sqrt(2.0 / 3.141592653589793) * x);
  const float xx = float(x * x);
  const float b = float(0.044715 * double(xx));
  const float c = float(1.0 + double(b));
  const float inner = float(double(a) * double(c));
  const float hx = float(0.5 * x);
  const float t = float(1.0 + tanh(double(inner)));
  return double(float(double(hx) * double(t)));
}

__global__ void hc_dgeglu_kernel(const float* __restrict__ g, const float* __restrict__ u, int n, float* __restrict__ o) {
  const int i = int(blockIdx.x * blockDim.x + threadIdx.x);
  if (i < n) o[i] = float(gelu_f32points(g[i]) * double(u[i]));
}

// Ordering key: value descending, then id ascending (runtime.ts:514-527);
// larger key = better, 0 = empty.
__device__ __forceinline__ uint64_t dkey(float v, uint32_t id) {
  uint32_t b = __float_as_uint(v);
  if (v == 0.0f) b = 0;
  const uint32_t ord = (v != v) ? 0u : ((b & 0x80000000u) ? ~b : (b | 0x80000000u));
  return (uint64_t(ord) << 32) | uint64_t(0xffffffffu - id);
}

// Top-k of n <= DT_MAXN entries (values with id = index, or ready keys), in
// one CTA, descending.  *d_k (device) or k.  Keys are unique apart from the
// empty key 0 (ids differ), so for k <= DT_SEL_MAX the k-th largest key is
// found by an 8-bit radix select (eight histogram passes over the keys held
// in registers), the keys at or above it are gathered and each is placed by
// its rank among them; larger k take a bitonic sort of all keys.
constexpr int DT_KPT = DT_MAXN / DT_THREADS;  // keys per thread
constexpr int DT_SEL_MAX = 64;
__global__ void __launch_bounds__(DT_THREADS) hc_dtopk_kernel(const float* __restrict__ vals,
                                                           const uint64_t* __restrict__ keys, int n, int k,
                                                           const int* __restrict__ d_k, int32_t* __restrict__ out_ids,
                                                           float* __restrict__ out_vals) {
  __shared__ uint64_t s[DT_MAXN];
  __shared__ int hist[256];
  __shared__ uint64_t s_prefix;
  __shared__ int s_rank, s_cnt;
  const int kk = d_k ? *d_k : k;
  auto emit = [&](int i, uint64_t key) {
    const uint32_t ord = uint32_t(key >> 32);
    const uint32_t bits = (ord & 0x80000000u) ? (ord & 0x7fffffffu) : ~ord;
    out_ids[i] = key ? int32_t(0xffffffffu - uint32_t(key)) : -1;
    out_vals[i] = key ? __uint_as_float(bits) : -INFINITY;
  };
  if (kk <= DT_SEL_MAX && kk < n) {
    uint64_t v[DT_KPT];
#pragma unroll
    for (int j = 0; j < DT_KPT; ++j) {
      const int i = int(threadIdx.x) + j * DT_THREADS;
      v[j] = i >= n ? 0ull : (keys ? keys[i] : dkey(vals[i], uint32_t(i)));
    }
    if (threadIdx.x == 0) {
      s_prefix = 0ull;
      s_rank = kk;  // rank of the wanted key among those matching the prefix
      s_cnt = 0;
    }
    uint64_t mask = 0ull;
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int i = int(threadIdx.x); i < 256; i += DT_THREADS) hist[i] = 0;
      __syncthreads();
      const uint64_t prefix = s_prefix;
#pragma unroll
      for (int j = 0; j < DT_KPT; ++j)
        if ((v[j] & mask) == prefix) atomicAdd(&hist[int(v[j] >> shift) & 255], 1);
      __syncthreads();
      if (threadIdx.x < 32) {  // warp 0: the digit where the count from the top reaches the rank
        const int lane = int(threadIdx.x);
        int c[8], tot = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {  // lane holds digits 255 - 8 lane - q (descending)
          c[q] = hist[255 - 8 * lane - q];
          tot += c[q];
        }
        int incl = tot;  // inclusive prefix over lanes (higher digits first)
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += y;
        }
        const int rank = s_rank;
        const int before = incl - tot;  // keys with a higher digit, over lower lanes
        if (before < rank && rank <= incl) {
          int acc = before, q = 0;
          while (q < 7 && acc + c[q] < rank) acc += c[q++];
          s_rank = rank - acc;
          s_prefix = prefix | (uint64_t(255 - 8 * lane - q) << shift);
        }
      }
      mask |= 0xffull << shift;
      __syncthreads();
    }
    const uint64_t kth = s_prefix;  // the kk-th largest key
    // gather the non-empty keys at or above it: kk of them, fewer when the
    // kk-th key is the empty one (the rest of the list is then empty)
#pragma unroll
    for (int j = 0; j < DT_KPT; ++j) {
      const int i = int(threadIdx.x) + j * DT_THREADS;
      if (i < n && v[j] >= kth && v[j] != 0ull) {
        const int slot = atomicAdd(&s_cnt, 1);
        if (slot < DT_SEL_MAX) s[slot] = v[j];
      }
    }
    __syncthreads();
    const int m = min(s_cnt, DT_SEL_MAX);
    for (int i = int(threadIdx.x); i < kk; i += DT_THREADS) {
      if (i >= m) {
        emit(i, 0ull);
        continue;
      }
      const uint64_t key = s[i];
      int r = 0;
      for (int j = 0; j < m; ++j) r += s[j] > key ? 1 : 0;
      emit(r, key);
    }
    return;
  }
  int np = 1;
  while (np < n) np <<= 1;
  for (int i = int(threadIdx.x); i < np; i += int(blockDim.x))
    s[i] = i >= n ? 0ull : (keys ? keys[i] : dkey(vals[i], uint32_t(i)));
  __syncthreads();
  for (int size = 2; size <= np; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = int(threadIdx.x); i < np; i += int(blockDim.x)) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;  // descending runs first: the final order is descending
          const uint64_t a = s[i], b = s[j];
          if (desc ? a < b : a > b) {
            s[i] = b;
            s[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = int(threadIdx.x); i < kk; i += int(blockDim.x)) emit(i, i < n ? s[i] : 0ull);
}

// maskedEmbeddingTopTokens (mtp-assistant-runner.ts:211-242): slot s of the
// top centroids' token lists (token_ordering[c * per + j]) scored by its
// embedding row . h -- the row dequantized bit-exactly from its row tile and
// one sequential f32 chain over the hidden index, as
// hp_matmul_dequantized_f32 on the gathered rows; ids outside the vocabulary
// get the empty key.  CTA = 32 slots: one chain warp (lane = slot) and four
// dequant warps that turn 256-block b of the 32 gathered rows into one half
// of a double buffer while the chain warp walks the other half (one barrier
// per block); every row's blocks are prefetched into L2 at the start.
constexpr int DS_DQ_WARPS = 4;
constexpr int DS_ROW = QK + 4;  // floats per staged row (16-byte reads by lane = slot hit distinct banks)
__global__ void __launch_bounds__(32 * (1 + DS_DQ_WARPS)) hc_dscores_kernel(
    const uint8_t* __restrict__ E, int type, int nb, int vocab, const int32_t* __restrict__ ordering, int per,
    const int32_t* __restrict__ c_ids, int slots, const float* __restrict__ h, uint64_t* __restrict__ keys) {
  extern __shared__ __align__(16) float ds_smem[];  // h [K], then rows [2][32][DS_ROW]
  __shared__ int toks[32];
  const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31);
  const int K = nb * QK;
  const int slot0 = int(blockIdx.x) * 32;
  if (warp == 0) {
    const int slot = slot0 + lane;
    int tok = -1;
    if (slot < slots) {
      const int c = c_ids[slot / per];
      tok = c >= 0 ? ordering[size_t(c) * per + slot % per] : -1;
      if (tok >= vocab) tok = -1;
    }
    toks[lane] = tok;
  }
  float* hs = ds_smem;
  float* ws = ds_smem + K;
  for (int i = int(threadIdx.x); i < K; i += int(blockDim.x)) hs[i] = h[i];
  __syncthreads();
  const size_t ub = type == TYPE_Q4_K ? Q4K_TILE_BLOCK_BYTES : Q6K_TILE_BLOCK_BYTES;
  const int dt = int(threadIdx.x) - 32;  // dequant thread index (< 0: the chain warp)
  if (dt >= 0) {
    // every (row, block): its 16-byte pieces at a 512-byte stride in the tile
    const int pieces = type == TYPE_Q4_K ? Q4K_CHUNKS : Q6K_CHUNKS;
    for (int task = dt; task < 32 * nb; task += 32 * DS_DQ_WARPS) {
      const int r = task & 31, b = task >> 5, tok = toks[r];
      if (tok < 0) continue;
      const uint8_t* tb = E + (size_t(tok / TILE) * nb + b) * ub + size_t(tok % TILE) * 16;
      for (int c = 0; c < pieces; ++c) asm volatile("prefetch.global.L2 [%0];" ::"l"(tb + size_t(c) * 512));
    }
  }
  auto fill = [&](int b, int buf) {
    float* wb = ws + buf * 32 * DS_ROW;
    for (int task = dt; task < 32 * 8; task += 32 * DS_DQ_WARPS) {  // (row, 32-element part)
      const int r = task >> 3, part = task & 7, tok = toks[r];
      float* o = wb + r * DS_ROW;
      if (tok < 0) continue;
      const uint8_t* tb = E + (size_t(tok / TILE) * nb + b) * ub;
      if (type == TYPE_Q4_K) q4k_dequant_chunk(tb, tok % TILE, part, o);
      else q6k_dequant_group(tb, tok % TILE, part, o);
    }
  };
  if (dt >= 0) fill(0, 0);
  __syncthreads();
  float sum = 0.0f;
  for (int b = 0; b < nb; ++b) {
    const int buf = b & 1;
    if (warp == 0) {
      const float4* wr = reinterpret_cast<const float4*>(ws + buf * 32 * DS_ROW + lane * DS_ROW);
      const float4* xc = reinterpret_cast<const float4*>(hs + b * QK);
#pragma unroll 8
      for (int i = 0; i < QK / 4; ++i) {
        const float4 a = wr[i], v = xc[i];
        sum = __fadd_rn(sum, __fmul_rn(a.x, v.x));
        sum = __fadd_rn(sum, __fmul_rn(a.y, v.y));
        sum = __fadd_rn(sum, __fmul_rn(a.z, v.z));
        sum = __fadd_rn(sum, __fmul_rn(a.w, v.w));
      }
    } else if (b + 1 < nb) {
      fill(b + 1, buf ^ 1);
    }
    __syncthreads();
  }
  if (warp == 0 && slot0 + lane < slots) keys[slot0 + lane] = toks[lane] >= 0 ? dkey(sum, uint32_t(toks[lane])) : 0ull;
}

// The step's inputs: [embedding ; hidden] into xin, the position and top-k.
__global__ void hc_dinputs_kernel(const float* __restrict__ emb, const float* __restrict__ hid, int n, float* xin,
                               int* d_pos, int position, int* d_k, int k) {
  const int i = int(blockIdx.x * blockDim.x + threadIdx.x);
  if (i < n) {
    xin[i] = emb[i];
    xin[n + i] = hid[i];
  }
  if (i == 0) {
    *d_pos = position;
    *d_k = k;
  }
}

}  // namespace
}  // namespace hc

namespace {

constexpr uint32_t kDraftMagic = 0x48504444u;  // "HPDD"

// One matrix of the head: its own copy of the resident row-tile bytes.
struct DraftMat {
  uint8_t* w = nullptr;
  size_t bytes = 0;
  int type = 0, nb = 0, rows = 0, rows_pad = 0;
};

struct DraftLayer {
  DraftMat w[HPC_DW_LAYER_COUNT];
  float* n[HPC_DN_LAYER_COUNT] = {};
  float scale = 1.0f;
  const float* kc = nullptr;
  const float* vc = nullptr;
};

}  // namespace

struct hpc_draft_s {
  uint32_t magic = kDraftMagic;
  int device = 0;
  hpc_draft_config cfg{};
  int per = 0;  // token_ordering entries per centroid
  DraftMat pre, post, cent, embd;
  float* out_norm = nullptr;
  int32_t* ordering = nullptr;
  std::vector<DraftLayer> layers;
  // workspace
  float *xin = nullptr, *x = nullptr, *a = nullptr, *q = nullptr, *att = nullptr, *o = nullptr, *r = nullptr,
        *nn = nullptr, *g = nullptr, *u = nullptr, *act = nullptr, *dn = nullptr, *h = nullptr, *post_out = nullptr,
        *cent_out = nullptr, *pm = nullptr, *pl = nullptr, *po = nullptr, *out_vals = nullptr, *c_vals = nullptr;
  int32_t *out_ids = nullptr, *c_ids = nullptr;
  uint64_t* keys = nullptr;
  int *d_pos = nullptr, *d_k = nullptr;
  cudaGraphExec_t graph = nullptr;
  std::vector<const void*> graph_kv;  // KV pointers the graph was captured with
};

static bool draft_valid(hpc_draft d) { return d && d->magic == kDraftMagic; }

static void draft_free(hpc_draft d) {
  for (DraftMat* m : {&d->pre, &d->post, &d->cent, &d->embd}) {
    cudaFree(m->w);
    *m = DraftMat{};
  }
  float** fs[] = {&d->out_norm, &d->xin, &d->x, &d->a, &d->q, &d->att,
                  &d->o, &d->r, &d->nn, &d->g, &d->u, &d->act, &d->dn, &d->h, &d->post_out, &d->cent_out,
                  &d->pm, &d->pl, &d->po, &d->out_vals, &d->c_vals};
  for (float** p : fs) {
    cudaFree(*p);
    *p = nullptr;
  }
  for (auto& L : d->layers) {
    for (DraftMat& m : L.w) {
      cudaFree(m.w);
      m = DraftMat{};
    }
    for (float*& p : L.n) cudaFree(p);
  }
  cudaFree(d->ordering);
  cudaFree(d->out_ids);
  cudaFree(d->c_ids);
  cudaFree(d->keys);
  cudaFree(d->d_pos);
  cudaFree(d->d_k);
  if (d->graph) cudaGraphExecDestroy(d->graph);
  d->graph = nullptr;
}

static void draft_invalidate(hpc_draft d) {
  if (d->graph) cudaGraphExecDestroy(d->graph);
  d->graph = nullptr;
}

// Matrix `which` of the draft head: its (input, rows) and its slot.
static int draft_matrix(hpc_draft d, int which, int layer, size_t* k, size_t* n, DraftMat** slot) {
  const hpc_draft_config& c = d->cfg;
  const size_t E = size_t(c.hidden), D = size_t(c.backbone), Hq = size_t(c.heads) * c.head_dim;
  if (which >= HPC_DW_PRE) {
    switch (which) {
      case HPC_DW_PRE: *k = 2 * D; *n = E; *slot = &d->pre; return HPC_OK;
      case HPC_DW_POST: *k = E; *n = D; *slot = &d->post; return HPC_OK;
      case HPC_DW_CENTROIDS: *k = E; *n = size_t(c.n_centroids); *slot = &d->cent; return HPC_OK;
      case HPC_DW_EMBD: *k = E; *n = size_t(c.vocab); *slot = &d->embd; return HPC_OK;
      default: return hpc_fail(HPC_ERR_ARG, "draft matrix id %d", which);
    }
  }
  if (layer < 0 || layer >= c.layers) return hpc_fail(HPC_ERR_ARG, "draft layer %d", layer);
  DraftLayer& L = d->layers[size_t(layer)];
  switch (which) {
    case HPC_DW_Q: *k = E; *n = Hq; break;
    case HPC_DW_O: *k = Hq; *n = E; break;
    case HPC_DW_GATE: case HPC_DW_UP: *k = E; *n = size_t(c.ffn); break;
    case HPC_DW_DOWN: *k = size_t(c.ffn); *n = E; break;
    default: return hpc_fail(HPC_ERR_ARG, "draft matrix id %d", which);
  }
  *slot = &L.w[which];
  return HPC_OK;
}

extern "C" {

int hpc_draft_create(const hpc_draft_config* cfg, hpc_draft* out) {
  if (!cfg || !out) return hpc_fail(HPC_ERR_ARG, "null pointer");
  const hpc_draft_config& c = *cfg;
  if (c.head_dim != 256 || c.heads < 1 || c.kv_heads < 1 || c.heads % c.kv_heads || c.layers < 1 ||
      c.hidden % 256 || c.backbone % 256 || c.ffn % 256 || c.context < 1 || c.context > 4096 ||
      c.context % 64 || c.n_centroids < 1 || c.n_centroids > 4096 || c.centroid_top_k < 1 ||
      c.centroid_top_k > c.n_centroids || c.max_top_k < 1 || c.max_top_k > 64 || c.vocab < 1 ||
      c.heads * c.head_dim % 4 || c.hidden > 8192 || c.backbone > 8192 || c.ffn > 65536)
    return hpc_fail(HPC_ERR_SHAPE, "draft head config");
  hpc_draft d = new hpc_draft_s();
  d->cfg = c;
  d->layers.resize(size_t(c.layers));
  cudaGetDevice(&d->device);
  const size_t E = size_t(c.hidden), D = size_t(c.backbone), Hq = size_t(c.heads) * c.head_dim, F = size_t(c.ffn);
  const size_t chunks = size_t(c.context) / hc::DA_CHUNK;
  const size_t G = size_t(c.heads / c.kv_heads);
  struct A {
    void** p;
    size_t bytes;
  } allocs[] = {
      {(void**)&d->xin, 4 * 2 * D}, {(void**)&d->x, 4 * E},    {(void**)&d->a, 4 * E},    {(void**)&d->q, 4 * Hq},
      {(void**)&d->att, 4 * Hq},    {(void**)&d->o, 4 * E},    {(void**)&d->r, 4 * E},    {(void**)&d->nn, 4 * E},
      {(void**)&d->g, 4 * F},       {(void**)&d->u, 4 * F},    {(void**)&d->act, 4 * F},  {(void**)&d->dn, 4 * E},
      {(void**)&d->h, 4 * E},       {(void**)&d->post_out, 4 * D}, {(void**)&d->cent_out, 4 * size_t(c.n_centroids)},
      {(void**)&d->pm, 4 * chunks * c.kv_heads * G}, {(void**)&d->pl, 4 * chunks * c.kv_heads * G},
      {(void**)&d->po, 4 * chunks * c.kv_heads * G * 256}, {(void**)&d->out_vals, 4 * 64},
      {(void**)&d->c_vals, 4 * size_t(c.centroid_top_k)}, {(void**)&d->out_ids, 4 * 64},
      {(void**)&d->c_ids, 4 * size_t(c.centroid_top_k)}, {(void**)&d->keys, 8 * size_t(hc::DT_MAXN)},
      {(void**)&d->d_pos, 4}, {(void**)&d->d_k, 4}, {(void**)&d->out_norm, 4 * E}};
  for (auto& a : allocs) {
    cudaError_t e = cudaMalloc(a.p, a.bytes);
    if (e != cudaSuccess) {
      draft_free(d);
      delete d;
      return hpc_cuda_fail(e, "cudaMalloc(draft workspace)");
    }
  }
  for (auto& L : d->layers)
    for (float*& p : L.n) {
      cudaError_t e = cudaMalloc(&p, 4 * E);
      if (e != cudaSuccess) {
        draft_free(d);
        delete d;
        return hpc_cuda_fail(e, "cudaMalloc(draft norms)");
      }
    }
  *out = d;
  return HPC_OK;
}

int hpc_draft_release(hpc_draft d) {
  if (!draft_valid(d)) return hpc_fail(HPC_ERR_ARG, "invalid draft head");
  draft_free(d);
  d->magic = 0;
  delete d;
  return HPC_OK;
}

int hpc_draft_set_matrix(hpc_draft d, int which, int layer, hpc_weight w) {
  if (!draft_valid(d)) return hpc_fail(HPC_ERR_ARG, "invalid draft head");
  if (!hpc_weight_valid(w)) return hpc_fail(HPC_ERR_ARG, "invalid weight handle");
  size_t k = 0, n = 0;
  DraftMat* slot = nullptr;
  int rc = draft_matrix(d, which, layer, &k, &n, &slot);
  if (rc != HPC_OK) return rc;
  if (w->input_size != k || w->row_count != n)
    return hpc_fail(HPC_ERR_SHAPE, "draft matrix %d: %zux%zu, expected %zux%zu", which, w->input_size, w->row_count,
                    k, n);
  if (slot->w && slot->bytes != w->bytes) {
    cudaFree(slot->w);
    slot->w = nullptr;
  }
  if (!slot->w) HPC_CK(cudaMalloc(&slot->w, w->bytes), "cudaMalloc(draft matrix)");
  // the resident row tiles, copied (the caller may release its handle)
  HPC_CK(cudaMemcpy(slot->w, w->d_data, w->bytes, cudaMemcpyDeviceToDevice), "draft matrix copy");
  slot->bytes = w->bytes;
  slot->type = w->type;
  slot->nb = w->nb;
  slot->rows = int(w->row_count);
  slot->rows_pad = int(w->rows_pad);
  draft_invalidate(d);
  return HPC_OK;
}

int hpc_draft_set_vector(hpc_draft d, int which, int layer, const float* host, size_t len) {
  if (!draft_valid(d)) return hpc_fail(HPC_ERR_ARG, "invalid draft head");
  if (!host) return hpc_fail(HPC_ERR_ARG, "null vector");
  const hpc_draft_config& c = d->cfg;
  float* dst = nullptr;
  size_t need = size_t(c.hidden);
  if (which == HPC_DN_OUTPUT) {
    dst = d->out_norm;
  } else {
    if (layer < 0 || layer >= c.layers || which < 0 || which >= HPC_DN_LAYER_COUNT)
      return hpc_fail(HPC_ERR_ARG, "draft vector %d of layer %d", which, layer);
    dst = d->layers[size_t(layer)].n[which];
    if (which == HPC_DN_Q) need = size_t(c.head_dim);
  }
  if (len != need) return hpc_fail(HPC_ERR_SHAPE, "draft vector %d: %zu values, expected %zu", which, len, need);
  HPC_CK(cudaMemcpy(dst, host, 4 * len, cudaMemcpyHostToDevice), "draft vector upload");
  return HPC_OK;
}

int hpc_draft_set_layer_scale(hpc_draft d, int layer, float scale) {
  if (!draft_valid(d)) return hpc_fail(HPC_ERR_ARG, "invalid draft head");
  if (layer < 0 || layer >= d->cfg.layers) return hpc_fail(HPC_ERR_ARG, "draft layer %d", layer);
  d->layers[size_t(layer)].scale = scale;
  draft_invalidate(d);
  return HPC_OK;
}

int hpc_draft_set_token_ordering(hpc_draft d, const int32_t* host, size_t len) {
  if (!draft_valid(d)) return hpc_fail(HPC_ERR_ARG, "invalid draft head");
  if (!host) return hpc_fail(HPC_ERR_ARG, "null ordering");
  const size_t per = len / size_t(d->cfg.n_centroids);
  if (per < 1 || per * size_t(d->cfg.centroid_top_k) > size_t(hc::DT_MAXN))
    return hpc_fail(HPC_ERR_SHAPE, "token ordering of %zu entries for %d centroids", len, d->cfg.n_centroids);
  cudaFree(d->ordering);
  d->ordering = nullptr;
  HPC_CK(cudaMalloc(&d->ordering, 4 * len), "cudaMalloc(token ordering)");
  HPC_CK(cudaMemcpy(d->ordering, host, 4 * len, cudaMemcpyHostToDevice), "token ordering upload");
  d->per = int(per);
  draft_invalidate(d);
  return HPC_OK;
}

int hpc_draft_set_target_kv(hpc_draft d, int layer, const float* d_key, const float* d_value) {
  if (!draft_valid(d)) return hpc_fail(HPC_ERR_ARG, "invalid draft head");
  if (layer < 0 || layer >= d->cfg.layers) return hpc_fail(HPC_ERR_ARG, "draft layer %d", layer);
  if (!d_key || !d_value) return hpc_fail(HPC_ERR_ARG, "null KV");
  d->layers[size_t(layer)].kc = d_key;
  d->layers[size_t(layer)].vc = d_value;
  return HPC_OK;
}

static int draft_enqueue(hpc_draft d, cudaStream_t st) {
  using namespace hc;
  const hpc_draft_config& c = d->cfg;
  const int E = c.hidden, D = c.backbone, Hq = c.heads * c.head_dim, F = c.ffn;
  // y = W x with hp_matmul_dequantized_f32's arithmetic (one sequential
  // chain per row over the bit-exactly dequantized weights)
  auto gemv = [&](const DraftMat& W, const float* x, float* y) -> int {
    HPC_CK(launch_dequant_matmul(W.type, W.w, W.nb, W.rows, W.rows_pad, x, W.nb * QK, 1, y, st), "draft gemv");
    return HPC_OK;
  };
  auto norm = [&](int mode, int n, const float* x, const float* y, const float* w1, const float* w2, float scale,
                  float* o1, float* o2) -> int {
    hc_dnorm_kernel<<<1, DN_THREADS, size_t(n) * 4, st>>>(mode, n, x, y, w1, w2, c.rms_eps, scale, o1, o2);
    HPC_CK(cudaGetLastError(), "draft norm");
    return HPC_OK;
  };
  int rc = gemv(d->pre, d->xin, d->x);
  if (rc != HPC_OK) return rc;
  const int pairs = int(std::floor(double(c.head_dim) * 0.25 / 2.0));
  const double theta_scale = std::pow(c.rope_theta, -2.0 / double(c.head_dim));
  const int G = c.heads / c.kv_heads, chunks = c.context / DA_CHUNK;
  for (int l = 0; l < c.layers; ++l) {
    DraftLayer& L = d->layers[size_t(l)];
    if ((rc = norm(0, E, d->x, nullptr, L.n[HPC_DN_ATTN], nullptr, 1.0f, d->a, nullptr)) != HPC_OK) return rc;
    if ((rc = gemv(L.w[HPC_DW_Q], d->a, d->q)) != HPC_OK) return rc;
    hc_dqrope_kernel<<<c.heads, 256, 0, st>>>(d->q, L.n[HPC_DN_Q], c.head_dim, d->d_pos, pairs, theta_scale, c.rms_eps);
    HPC_CK(cudaGetLastError(), "draft q norm / rope");
    {
      static std::atomic<uint64_t> attr{0};
      const cudaError_t ea = once_per_current_device(attr, [] {
        return cudaFuncSetAttribute(hc_dattn_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(dattn_smem_floats(64) * 4));
      });
      HPC_CK(ea, "draft attention attributes");
    }
    hc_dattn_partial_kernel<<<dim3(chunks, c.kv_heads), 256, dattn_smem_floats(G) * 4, st>>>(
        d->q, L.kc, L.vc, d->d_pos, c.heads, c.kv_heads, d->pm, d->pl, d->po);
    HPC_CK(cudaGetLastError(), "draft attention");
    hc_dattn_combine_kernel<<<c.heads, 256, 0, st>>>(d->pm, d->pl, d->po, d->d_pos, c.heads, c.kv_heads, d->att);
    HPC_CK(cudaGetLastError(), "draft attention combine");
    if ((rc = gemv(L.w[HPC_DW_O], d->att, d->o)) != HPC_OK) return rc;
    if ((rc = norm(1, E, d->x, d->o, L.n[HPC_DN_POST_ATTN], L.n[HPC_DN_FFN], 1.0f, d->r, d->nn)) != HPC_OK) return rc;
    if ((rc = gemv(L.w[HPC_DW_GATE], d->nn, d->g)) != HPC_OK) return rc;
    if ((rc = gemv(L.w[HPC_DW_UP], d->nn, d->u)) != HPC_OK) return rc;
    hc_dgeglu_kernel<<<(F + 255) / 256, 256, 0, st>>>(d->g, d->u, F, d->act);
    HPC_CK(cudaGetLastError(), "draft geglu");
    if ((rc = gemv(L.w[HPC_DW_DOWN], d->act, d->dn)) != HPC_OK) return rc;
    if ((rc = norm(2, E, d->r, d->dn, L.n[HPC_DN_POST_FFW], nullptr, L.scale, d->x, nullptr)) != HPC_OK) return rc;
  }
  if ((rc = norm(0, E, d->x, nullptr, d->out_norm, nullptr, 1.0f, d->h, nullptr)) != HPC_OK) return rc;
  if ((rc = gemv(d->post, d->h, d->post_out)) != HPC_OK) return rc;
  if ((rc = gemv(d->cent, d->h, d->cent_out)) != HPC_OK) return rc;
  hc_dtopk_kernel<<<1, DT_THREADS, 0, st>>>(d->cent_out, nullptr, c.n_centroids, c.centroid_top_k, nullptr, d->c_ids,
                                         d->c_vals);
  HPC_CK(cudaGetLastError(), "draft centroid top-k");
  const int slots = c.centroid_top_k * d->per;
  const size_t ds_bytes = (size_t(E) + 2 * 32 * DS_ROW) * 4;
  {
    static std::atomic<uint64_t> attr{0};
    const cudaError_t ea = once_per_current_device(attr, [] {
      return cudaFuncSetAttribute(hc_dscores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int((8192 + 2 * 32 * DS_ROW) * 4));
    });
    HPC_CK(ea, "draft token scores attributes");
  }
  hc_dscores_kernel<<<(slots + 31) / 32, 32 * (1 + DS_DQ_WARPS), ds_bytes, st>>>(
      d->embd.w, d->embd.type, d->embd.nb, c.vocab, d->ordering, d->per, d->c_ids, slots, d->h, d->keys);
  HPC_CK(cudaGetLastError(), "draft token scores");
  hc_dtopk_kernel<<<1, DT_THREADS, 0, st>>>(nullptr, d->keys, slots, 0, d->d_k, d->out_ids, d->out_vals);
  HPC_CK(cudaGetLastError(), "draft token top-k");
  return HPC_OK;
}

int hpc_draft_step(hpc_draft d, const float* d_embedding, const float* d_hidden, int position, size_t top_k,
                   float* d_post_out, int32_t* d_ids, float* d_vals, void* stream) {
  if (!draft_valid(d)) return hpc_fail(HPC_ERR_ARG, "invalid draft head");
  const hpc_draft_config& c = d->cfg;
  if (!d_embedding || !d_hidden || !d_post_out || !d_ids || !d_vals) return hpc_fail(HPC_ERR_ARG, "null pointer");
  if (position < 0 || position >= c.context) return hpc_fail(HPC_ERR_SHAPE, "draft position %d", position);
  if (top_k < 1 || top_k > size_t(c.max_top_k)) return hpc_fail(HPC_ERR_SHAPE, "draft top-k %zu", top_k);
  if (!d->pre.w || !d->post.w || !d->cent.w || !d->embd.w || !d->ordering)
    return hpc_fail(HPC_ERR_ARG, "draft head weights not loaded");
  std::vector<const void*> kv;
  for (auto& L : d->layers) {
    for (const DraftMat& w : L.w)
      if (!w.w) return hpc_fail(HPC_ERR_ARG, "draft layer weights not loaded");
    if (!L.kc || !L.vc) return hpc_fail(HPC_ERR_ARG, "draft target KV not set");
    kv.push_back(L.kc);
    kv.push_back(L.vc);
  }
  if (top_k > size_t(c.centroid_top_k) * size_t(d->per))
    return hpc_fail(HPC_ERR_SHAPE, "draft top-k %zu above the %d candidate tokens", top_k,
                    c.centroid_top_k * d->per);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int D = c.backbone;
  hc::hc_dinputs_kernel<<<(D + 255) / 256, 256, 0, st>>>(d_embedding, d_hidden, D, d->xin, d->d_pos, position, d->d_k,
                                                      int(top_k));
  HPC_CK(cudaGetLastError(), "draft inputs");
  if (!d->graph || d->graph_kv != kv) {
    draft_invalidate(d);
    cudaStream_t cs;
    HPC_CK(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking), "capture stream");
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
    int rc = HPC_OK;
    if (e == cudaSuccess) {
      rc = draft_enqueue(d, cs);
      e = cudaStreamEndCapture(cs, &g);
    }
    cudaStreamDestroy(cs);
    if (rc != HPC_OK) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return hpc_cuda_fail(e, "draft graph capture");
    e = cudaGraphInstantiate(&d->graph, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return hpc_cuda_fail(e, "draft graph instantiate");
    d->graph_kv = kv;
  }
  HPC_CK(cudaGraphLaunch(d->graph, st), "draft graph launch");
  HPC_CK(cudaMemcpyAsync(d_post_out, d->post_out, 4 * size_t(D), cudaMemcpyDeviceToDevice, st), "draft post copy");
  HPC_CK(cudaMemcpyAsync(d_ids, d->out_ids, 4 * top_k, cudaMemcpyDeviceToDevice, st), "draft ids copy");
  HPC_CK(cudaMemcpyAsync(d_vals, d->out_vals, 4 * top_k, cudaMemcpyDeviceToDevice, st), "draft values copy");
  return HPC_OK;
}

}  // extern "C"
