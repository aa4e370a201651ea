// hc_decode.cu -- the per-layer decoder math around the quantized matmuls.
//
// Restates forwardAttentionLayer / forwardFfn / forwardOutput of the WASM
// provider (packages/engine/src/runner/wasm/layers.ts:161-473) as CUDA
// kernels.  The reference computes in JavaScript numbers (f64) and rounds to
// f32 at stores and Math.fround; the kernels keep those rounding points:
//   * RMSNorm (layers.ts:871-885): f64 sum of squares, f64 scale
//     1/sqrt(ss/n + eps), product x*scale*w in f64, stored as f32;
//   * RoPE NeoX (layers.ts:990-1033): theta chain fround(theta*base^(-2/n)),
//     cos/sin in f64, each product rounded to f32;
//   * attention (lib.rs:539-654 via layers.ts:304-334): query rounded to f16
//     with the Rust codec, scale 1, causal mask, f64 exp; the output is cast
//     through the TS f16 codec (castF16Rows, layers.ts:982-988);
//   * GEGLU (layers.ts:450-456, gelu 1062-1076): tanh-GELU with f16 round
//     trips of its input and output, product rounded to f32.
// Parallel reductions (sums of squares, dot products, softmax across KV
// chunks) run in a different order than the reference's sequential loops, so
// results agree to f32/f64 rounding, not bit for bit.
//
// Every kernel is launched with programmatic dependent launch: it signals its
// dependents early and waits (griddepcontrol.wait) before touching memory the
// previous kernel writes.
#include <cmath>
#include <utility>

#include <cuda_fp16.h>

#include "hc_bulk.cuh"
#include "hc_common.cuh"
#include "hc_decmath.cuh"
#include "hc_decode.cuh"
#include "hc_kernels.cuh"
#include "hc_q8.cuh"
#include "hc_unpack.cuh"

namespace hc {

// ---- RoPE table -------------------------------------------------------------------

// cos/sin of the NeoX RoPE angles for each token (layers.ts:1012-1030):
// theta_0 = position, theta_{i+1} = fround(theta_i * base^(-2/ndims)), cos
// and sin in f64.  The rows come from a table computed once on the host with
// the C library's cos/sin (the functions the reference's Math.cos/Math.sin
// stand for); a position past the table is computed here instead (the theta
// chain serially by one thread, the cos/sin in parallel).  One CTA per token.
__global__ void hc_rope_gather_kernel(const int32_t* __restrict__ pos, int half, const double* __restrict__ cos_tab,
                                      const double* __restrict__ sin_tab, int table_rows, double theta_scale,
                                      double* __restrict__ cos_t, double* __restrict__ sin_t) {
  __shared__ double theta[512];
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x, p = pos[m];
  if (p >= 0 && p < table_rows) {
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      cos_t[size_t(m) * half + i] = cos_tab[size_t(p) * half + i];
      sin_t[size_t(m) * half + i] = sin_tab[size_t(p) * half + i];
    }
    return;
  }
  if (threadIdx.x == 0) {
    double th = double(p);
    for (int i = 0; i < half; ++i) {
      theta[i] = th;
      th = double(float(th * theta_scale));
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    cos_t[size_t(m) * half + i] = cos(theta[i]);
    sin_t[size_t(m) * half + i] = sin(theta[i]);
  }
}

// ---- embedding --------------------------------------------------------------------

// Dequantizes element e of row `row` from the tile layout (bit-exact to
// dequantize_q6_k / dequantize_q4_k, lib.rs:1709-1744 / 1630-1664).
__device__ __forceinline__ float tile_elem(const uint8_t* w, int type, int nb, int row, int e) {
  const int b = e >> 8, r = e & 255, lane = row & 31;
  if (type == TYPE_Q6_K) {
    const uint8_t* unit = w + (size_t(row >> 5) * nb + b) * Q6K_TILE_BLOCK_BYTES;
    const int s16 = r >> 4, within = r & 15;
    const int j = (within & 7) >> 1, i = ((within >> 3) & 1) | ((within & 1) << 1);
    const int s = s16 & 7, hi = s16 >> 3;
    const uint8_t nb_byte = unit[size_t(s) * 512 + lane * 16 + j * 4 + i];
    const int h = 2 * s + (j >> 1);
    const uint8_t hw_byte = unit[size_t(8 + (h >> 2)) * 512 + lane * 16 + (h & 3) * 4 + i];
    const uint32_t lo = hi ? (nb_byte >> 4) : (nb_byte & 15);
    const uint32_t hb = (hw_byte >> (2 * (j & 1) + 4 * hi)) & 3;
    const int q = int(lo | (hb << 4)) - 32;
    const int sc = int(int8_t(unit[size_t(12) * 512 + lane * 16 + s16]));
    const float d = f16_bits_to_f32(reinterpret_cast<const uint16_t*>(unit + Q6K_DPLANE_OFFSET)[lane]);
    return __fmul_rn(__fmul_rn(d, float(sc)), float(q));
  }
  const uint8_t* unit = w + (size_t(row >> 5) * nb + b) * Q4K_TILE_BLOCK_BYTES;
  const uint4 hv = *reinterpret_cast<const uint4*>(unit + lane * 16);
  const Q4KHeader hd = q4k_header(hv);
  const int p = r >> 6, within64 = r & 63, half = within64 >> 5, l8 = within64 & 31;
  const int l = l8 & 7, i = l8 >> 3;
  const uint8_t byte = unit[size_t(1 + 2 * p + (l >> 2)) * 512 + lane * 16 + (l & 3) * 4 + i];
  const int g = 2 * p + half;
  const uint32_t q = half ? (byte >> 4) : (byte & 15);
  return __fsub_rn(__fmul_rn(__fmul_rn(hd.d, float(hd.sc(g))), float(q)), __fmul_rn(hd.dmin, float(hd.mn(g))));
}

// prepareInput (layers.ts:54-67): hidden = fround(embedding_row * sqrt(D)).
__global__ void hc_embed_kernel(const uint8_t* __restrict__ w, int type, int nb, int vocab, const int32_t* __restrict__ ids,
                             float* __restrict__ hidden, int D, double scale, int* __restrict__ err) {
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.x;
  const int row = ids[m];
  if (row < 0 || row >= vocab) {
    if (threadIdx.x == 0 && err) atomicExch(err, 2);
    return;
  }
  for (int e = threadIdx.x; e < D; e += blockDim.x)
    hidden[size_t(m) * D + e] = float(double(tile_elem(w, type, nb, row, e)) * scale);
}

// ---- norms + quantize ----------------------------------------------------------------

// One CTA of D/8 threads per column (thread t owns elements 8t..8t+7; warp w
// owns 256-block w).  Mode RESID: h = x + rmsnorm(y, w_post) is stored to
// x_out (the residual stream, layers.ts:359-363 / 471; x_out may be x), then
// n = rmsnorm(h, w_pre); otherwise n = rmsnorm(x, w_pre).  n is quantized to
// Q8_K for the next matmul; if n_out != nullptr it is also stored as f32.
template <bool RESID>
__global__ void hc_norm_quant_kernel(const float* x, float* x_out, const float* __restrict__ y,
                                  const float* __restrict__ w_post, const float* __restrict__ w_pre, double eps, int D,
                                  Q8Buf q, float* __restrict__ n_out) {
  __shared__ double scratch[32];
  __shared__ __align__(16) uint8_t stage[32][256];
  pdl_trigger();
  const int m = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int warps = blockDim.x >> 5;
  // the norm weights are not written during the step: load them before the
  // wait, so only the activation loads sit behind it
  float wq[8], wp[8];
  load8(w_pre + 8 * t, wq);
  if (RESID) load8(w_post + 8 * t, wp);
  pdl_wait();
  float h[8], yv[8];
  load8(x + size_t(m) * D + 8 * t, h);
  if (RESID) load8(y + size_t(m) * D + 8 * t, yv);
  if (RESID) {
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += double(yv[i]) * double(yv[i]);
    ss = block_sum_d(ss, scratch, warps);
    const double sc = 1.0 / sqrt(ss / double(D) + eps);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float pn = float((double(yv[i]) * sc) * double(wp[i]));
      h[i] = h[i] + pn;
    }
    float4* xo = reinterpret_cast<float4*>(x_out + size_t(m) * D + 8 * t);
    xo[0] = make_float4(h[0], h[1], h[2], h[3]);
    xo[1] = make_float4(h[4], h[5], h[6], h[7]);
  }
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += double(h[i]) * double(h[i]);
  ss = block_sum_d(ss, scratch, warps);
  const double sc = 1.0 / sqrt(ss / double(D) + eps);
  float n[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) n[i] = float((double(h[i]) * sc) * double(wq[i]));
  if (n_out) {
    float4* no = reinterpret_cast<float4*>(n_out + size_t(m) * D + 8 * t);
    no[0] = make_float4(n[0], n[1], n[2], n[3]);
    no[1] = make_float4(n[4], n[5], n[6], n[7]);
  }
  q8k_block_warp(n, lane, stage[warp], q8_rec_a(q, m, warp), q8_rec_b(q, m, warp));
}

// ---- attention ------------------------------------------------------------------------

// Split-KV decode attention (flash-decoding form of hp_gqa_attention_f32,
// lib.rs:539-654, on the compacted full-attention range [0, pos+1)), with the
// QK-norm / RoPE of the queries and the write of this step's K/V rows
// (forwardAttentionLayer, layers.ts:201-268, 887-911) folded in.  Grid
// (chunks, KVH); a CTA serves all M tokens x (H/KVH) query heads of one KV
// head over one ATT_CHUNK-token slice of the cache.  Warp 0 issues bulk
// copies of the slice (ATT_CHUNK K rows and ATT_CHUNK V rows of 1 KB each)
// into padded shared-memory rows (bank-conflict-free reads),
// completing on an mbarrier.  A slice that holds none of this step's new
// rows (every chunk but the one or two around pos) was written by earlier
// steps, so its copies are issued before griddepcontrol.wait and overlap the
// kernels ahead of attention.  Then the queries are normed, rotated and
// rounded to f16 with the Rust codec (lib.rs:590-597) -- one warp per query
// vector -- the CTA holding a new row of an own-KV layer computes it (cache
// and staged copy), and scores (scale 1, causal), a local
// softmax (max, sum of f64 exp) and the partial output p*v are written for
// the combine kernel.
constexpr int ATT_KSTRIDE = 256 + 4;        // floats per staged K row
constexpr int ATT_QB = 8;                   // general wide form: queries per thread per output pass
constexpr int ATT_QBS = 4;                  // general wide form: queries per thread per score pass
// The wide form (more than four query vectors per KV head) runs twice the
// threads: its ~155 KB of staged rows and queries hold one CTA per SM, and
// eight warps there left the scheduler idle (44% issue, latency-bound).
constexpr int ATT_WIDE_THREADS = 2 * ATT_THREADS;

// Wide form: QS query slots per thread in the score pass (ATT_WIDE_THREADS /
// ATT_CHUNK query lanes) and PB per half of the CTA in the output pass.  The
// loops cover any NQ; sized to NQ, a thread idles at most one score slot and
// no output slot (a slot past NQ still issues its instructions).
template <bool WIDE, int QS = ATT_QBS, int PB = ATT_QB>
__global__ void __launch_bounds__(WIDE ? ATT_WIDE_THREADS : ATT_THREADS) hc_attn_partial_kernel(
    const float* __restrict__ q, const float* __restrict__ kraw, const float* __restrict__ vraw,
    const float* __restrict__ qnw, const float* __restrict__ knw, const double* __restrict__ cos_t,
    const double* __restrict__ sin_t, double eps, int own_kv, float* __restrict__ kc, float* __restrict__ vc,
    const int32_t* __restrict__ pos, int M, int H, int KVH, int cap, float scale, float* __restrict__ part_m,
    float* __restrict__ part_l, float* __restrict__ part_o, int* __restrict__ err) {
  constexpr int HD = 256, CH = ATT_CHUNK;
  static_assert(ATT_THREADS == HD, "thread d owns V row d");
  extern __shared__ __align__(16) float sm[];
  const int chunk = blockIdx.x, kvh = blockIdx.y;
  const int G = H / KVH, NQ = M * G;
  float* ks = sm;                     // [CH][ATT_KSTRIDE]
  float* vs = ks + CH * ATT_KSTRIDE;  // [CH][ATT_KSTRIDE]
  float* qs = vs + CH * ATT_KSTRIDE;  // [NQ][HD]
  float* ps = qs + NQ * HD;           // [NQ][CH]
  pdl_trigger();
  // pos is written before the step starts (not by a kernel of this step)
  int maxpos = 0;
  bool fresh = false;  // does the slice hold a row written in this step?
  const int t0 = chunk * CH;
  for (int i = 0; i < M; ++i) {
    const int p = pos[i];
    maxpos = max(maxpos, p);
    fresh |= (p >= t0 && p < t0 + CH);
  }
  const int count = min(cap, maxpos + 1);
  if (t0 >= count) {
    pdl_wait();
    return;
  }
  const int nt = min(CH, count - t0);
  // Every row of the slice is copied before the wait (cap % CH == 0 keeps
  // the copies of the last, partial chunk inside the cache) with 16-byte
  // asynchronous copies spread over all threads (a warp copies 512
  // contiguous bytes of a row).  Rows this step writes (the tokens at pos)
  // may be stale in that copy; they are replaced below, after the copies
  // have landed.
  {
    constexpr int PIECES = HD * 4 / 16;  // 16-byte pieces per row
    // when there are fewer query vectors than warps, the warps that prepare
    // the queries issue no copies: their q loads after the wait then do not
    // queue behind this slice's copies
    const int nw = int(blockDim.x >> 5), nq = M * (H / KVH), cw0 = nq < nw ? nq : 0;
    const int ncp = (nw - cw0) * 32;
    if (int(threadIdx.x >> 5) >= cw0)
      for (int i = int(threadIdx.x) - cw0 * 32; i < CH * PIECES; i += ncp) {
        const int t = i / PIECES, c = i % PIECES;
        const size_t row = (size_t(t0 + t) * KVH + kvh) * HD + 4 * c;
        cp_async16(ks + t * ATT_KSTRIDE + 4 * c, kc + row);
        cp_async16(vs + t * ATT_KSTRIDE + 4 * c, vc + row);
      }
    cp_async_commit();
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  // the QK-norm weights are not written during the step
  float qw[8], kw[8];
  load8(qnw + 8 * lane, qw);
  if (own_kv && fresh) load8(knw + 8 * lane, kw);
  pdl_wait();
  // queries of this KV head's G heads for every token: QK-norm + RoPE (the
  // token's row of the cos/sin tables), rounded with the Rust f16 codec
  // (lib.rs:590-597); one warp per vector
  for (int qi = warp; qi < NQ; qi += warps) {
    const int m = qi / G, h = kvh * G + qi % G;
    float x[8];
    double c8[8], s8[8];
    load8(q + (size_t(m) * H + h) * HD + 8 * lane, x);
    load_rope8(cos_t + size_t(m) * (HD / 2), sin_t + size_t(m) * (HD / 2), lane, c8, s8);
    head_norm_rope(x, qw, true, true, c8, s8, eps, lane);
#pragma unroll
    for (int i = 0; i < 8; ++i) qs[qi * HD + 8 * lane + i] = round_f16_rust(x[i]);
  }
  cp_async_wait_all();
  __syncthreads();  // every thread's copies of the slice have landed
  // This step's K/V rows in the slice replace the staged copies.  Own-KV
  // layer: computed here (key: K-norm + RoPE; value: unweighted norm;
  // layers.ts:241-268) and written to the cache (layers.ts:887-911).
  // Shared-KV layer: read from the cache, where the source layer's attention
  // launch earlier in the step wrote them.
  if (fresh) {
    for (int job = warp; job < 2 * M; job += warps) {
      const int m = job >> 1, isv = job & 1, p = pos[m];
      if (p < t0 || p >= t0 + CH) continue;
      float* cache = (isv ? vc : kc) + (size_t(p % cap) * KVH + kvh) * HD + 8 * lane;
      float x[8];
      if (own_kv) {
        double c8[8], s8[8];
        load8((isv ? vraw : kraw) + (size_t(m) * KVH + kvh) * HD + 8 * lane, x);
        if (!isv) load_rope8(cos_t + size_t(m) * (HD / 2), sin_t + size_t(m) * (HD / 2), lane, c8, s8);
        head_norm_rope(x, kw, !isv, !isv, c8, s8, eps, lane);
        reinterpret_cast<float4*>(cache)[0] = make_float4(x[0], x[1], x[2], x[3]);
        reinterpret_cast<float4*>(cache)[1] = make_float4(x[4], x[5], x[6], x[7]);
      } else {
        load8(cache, x);
      }
      float* staged = (isv ? vs : ks) + (p - t0) * ATT_KSTRIDE + 8 * lane;
#pragma unroll
      for (int i = 0; i < 8; ++i) staged[i] = x[i];
    }
  }
  __syncthreads();
  // scores.  One KV head's query vectors for one token (NQ <= 4): thread per
  // (query, token); a warp shares the query (broadcast reads) and walks 32
  // padded K rows.  Wider steps: thread (token t = tid % CH, query lane qg =
  // tid / CH) computes the dots of queries qg, qg + QL, ... (QS per pass)
  // with token t, so each 16-byte piece of its K row is read once
  // for all of them.  Both forms keep the same order inside a dot (four lanes
  // of partial sums, then (x + y) + (z + w)), so a dot does not depend on how
  // many tokens the step carries.
  if (!WIDE) {
    for (int pr = threadIdx.x; pr < NQ * CH; pr += blockDim.x) {
      const int qi = pr / CH, t = pr % CH;
      const float4* qv = reinterpret_cast<const float4*>(qs + qi * HD);
      const float4* kv = reinterpret_cast<const float4*>(ks + t * ATT_KSTRIDE);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 16
      for (int j = 0; j < HD / 4; ++j) {
        const float4 a = qv[j], b = kv[j];
        acc.x = fmaf(a.x, b.x, acc.x);
        acc.y = fmaf(a.y, b.y, acc.y);
        acc.z = fmaf(a.z, b.z, acc.z);
        acc.w = fmaf(a.w, b.w, acc.w);
      }
      const float dot = (acc.x + acc.y) + (acc.z + acc.w);
      const int m = qi / G;
      ps[pr] = (t < nt && t0 + t <= pos[m]) ? dot * scale : -INFINITY;
    }
  } else {
    constexpr int QL = ATT_WIDE_THREADS / CH;  // query lanes
    const int t = int(threadIdx.x) % CH, qg = int(threadIdx.x) / CH;
    const float4* kv = reinterpret_cast<const float4*>(ks + t * ATT_KSTRIDE);
    for (int q0 = qg; q0 < NQ; q0 += QL * QS) {
      float4 acc[QS];
#pragma unroll
      for (int u = 0; u < QS; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
      for (int j = 0; j < HD / 4; ++j) {
        const float4 b = kv[j];
#pragma unroll
        for (int u = 0; u < QS; ++u) {
          if (q0 + QL * u < NQ) {
            const float4 a = reinterpret_cast<const float4*>(qs + (q0 + QL * u) * HD)[j];
            acc[u].x = fmaf(a.x, b.x, acc[u].x);
            acc[u].y = fmaf(a.y, b.y, acc[u].y);
            acc[u].z = fmaf(a.z, b.z, acc[u].z);
            acc[u].w = fmaf(a.w, b.w, acc[u].w);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < QS; ++u) {
        const int qi = q0 + QL * u;
        if (qi < NQ) {
          const float dot = (acc[u].x + acc[u].y) + (acc[u].z + acc[u].w);
          ps[qi * CH + t] = (t < nt && t0 + t <= pos[qi / G]) ? dot * scale : -INFINITY;
        }
      }
    }
  }
  __syncthreads();
  // local softmax: warp per query
  for (int qi = warp; qi < NQ; qi += warps) {
    float mx = -INFINITY;
    for (int t = lane; t < CH; t += 32) mx = fmaxf(mx, ps[qi * CH + t]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.0f;
    for (int t = lane; t < CH; t += 32) {
      const float sc = ps[qi * CH + t];
      const float p = (sc == -INFINITY) ? 0.0f : float(exp(double(sc - mx)));
      ps[qi * CH + t] = p;
      sum += p;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == 0) {
      const size_t o = (size_t(chunk) * KVH + kvh) * NQ + qi;
      part_m[o] = mx;
      part_l[o] = sum;
    }
  }
  __syncthreads();
  // partial outputs: thread d walks column d of the staged V rows (a warp
  // reads 32 consecutive floats of a row) and serves four queries per pass
  // (NQ <= 4) or PB (wider steps, where the two halves of the CTA take
  // alternate passes); the probabilities are broadcast reads
  const int d = threadIdx.x & (HD - 1);
  if (!WIDE) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int j = 0; j < CH / 4; ++j) {
      const float b[4] = {vs[(4 * j) * ATT_KSTRIDE + d], vs[(4 * j + 1) * ATT_KSTRIDE + d],
                          vs[(4 * j + 2) * ATT_KSTRIDE + d], vs[(4 * j + 3) * ATT_KSTRIDE + d]};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (u < NQ) {
          const float4 a = reinterpret_cast<const float4*>(ps + u * CH)[j];
          acc[u] += a.x * b[0] + a.y * b[1] + a.z * b[2] + a.w * b[3];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (u < NQ) part_o[((size_t(chunk) * KVH + kvh) * NQ + u) * HD + d] = acc[u];
    return;
  }
  for (int qg = int(threadIdx.x / HD) * PB; qg < NQ; qg += (ATT_WIDE_THREADS / HD) * PB) {
    float acc[PB];
#pragma unroll
    for (int u = 0; u < PB; ++u) acc[u] = 0.f;
#pragma unroll 2
    for (int j = 0; j < CH / 4; ++j) {
      const float b[4] = {vs[(4 * j) * ATT_KSTRIDE + d], vs[(4 * j + 1) * ATT_KSTRIDE + d],
                          vs[(4 * j + 2) * ATT_KSTRIDE + d], vs[(4 * j + 3) * ATT_KSTRIDE + d]};
#pragma unroll
      for (int u = 0; u < PB; ++u) {
        if (qg + u < NQ) {
          const float4 a = reinterpret_cast<const float4*>(ps + (qg + u) * CH)[j];
          acc[u] += a.x * b[0] + a.y * b[1] + a.z * b[2] + a.w * b[3];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < PB; ++u)
      if (qg + u < NQ) part_o[((size_t(chunk) * KVH + kvh) * NQ + qg + u) * HD + d] = acc[u];
  }
}

// Combines the chunk partials of one (token, head): global max, rescaled
// sums, division, the TS f16 cast (castF16Rows), then the head's 256 values
// -- exactly Q8_K block h of the token's attention vector -- are quantized
// for the output projection.  Grid (M, H), thread d = head dimension.
__global__ void __launch_bounds__(256) hc_attn_combine_kernel(const float* __restrict__ part_m,
                                                           const float* __restrict__ part_l,
                                                           const float* __restrict__ part_o,
                                                           const int32_t* __restrict__ pos, int M, int H, int KVH,
                                                           int cap, Q8Buf q, float* __restrict__ attn_out) {
  constexpr int HD = 256, CH = ATT_CHUNK, MAXC = 4096 / ATT_CHUNK;
  __shared__ float wch[MAXC];
  __shared__ double red[8];
  __shared__ float vec[HD];
  __shared__ __align__(16) uint8_t stage[256];
  pdl_trigger();
  const int m = blockIdx.x, h = blockIdx.y, d = threadIdx.x, lane = d & 31, warp = d >> 5;
  const int G = H / KVH, NQ = M * G, kvh = h / G, qi = m * G + h % G;
  // pos is written before the step starts (not by a kernel of this step)
  int maxpos = 0;
  for (int i = 0; i < M; ++i) maxpos = max(maxpos, pos[i]);
  const int count = min(cap, maxpos + 1);
  const int nch = (count + CH - 1) / CH;
  pdl_wait();
  // Every load is issued up front: the chunk maxima and sums (thread d <
  // nch) and dimension d of all nch partial outputs (index clamped to the
  // last chunk; chunks >= nch get weight 0 below).
  float mc = -INFINITY, lc = 0.0f;
  if (d < nch) {
    mc = part_m[(size_t(d) * KVH + kvh) * NQ + qi];
    lc = part_l[(size_t(d) * KVH + kvh) * NQ + qi];
  }
  const float* po = part_o + (size_t(kvh) * NQ + qi) * HD + d;
  const size_t cstride = size_t(KVH) * NQ * HD;
  float v[MAXC];
#pragma unroll
  for (int i = 0; i < MAXC; ++i) v[i] = po[size_t(min(i, nch - 1)) * cstride];
  // chunk maxima -> global max
  float mx = mc;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) red[warp] = double(mx);
  __syncthreads();
  float gmax = -INFINITY;
  for (int w = 0; w < 8; ++w) gmax = fmaxf(gmax, float(red[w]));
  __syncthreads();
  // chunk weights and the total normalizer
  double lw = 0.0;
  if (d < MAXC) {
    const float w = (d >= nch || mc == -INFINITY) ? 0.0f : float(exp(double(mc - gmax)));
    wch[d] = w;
    lw = double(w) * double(lc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, off);
  if (lane == 0) red[warp] = lw;
  __syncthreads();
  double l = 0.0;
  for (int w = 0; w < 8; ++w) l += red[w];
  // weighted sum over chunks for dimension d, in chunk order
  float o = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) o += wch[i] * v[i];
  const float n = round_f16_ts(float(double(o) / l));
  vec[d] = n;
  if (attn_out) attn_out[(size_t(m) * H + h) * HD + d] = n;
  __syncthreads();
  if (warp == 0) {
    float v8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v8[i] = vec[8 * lane + i];
    q8k_block_warp(v8, lane, stage, q8_rec_a(q, m, h), q8_rec_b(q, m, h));
  }
}

// ---- GEGLU ----------------------------------------------------------------------------

// act = fround(gelu(gate) * up), quantized for the down projection.  One CTA
// per 256-block of one column, thread t = element t: the f64 tanh of the
// GELU (~1k cycles) runs once per thread, all blocks in parallel; warp 0 then
// quantizes the block.  Grid (F/256, M).
__global__ void __launch_bounds__(256) hc_geglu_quant_kernel(const float* __restrict__ gate, const float* __restrict__ up,
                                                          int F, Q8Buf q, float* __restrict__ act_out) {
  __shared__ float vals[256];
  __shared__ __align__(16) uint8_t stage[256];
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.y, b = blockIdx.x, t = threadIdx.x, lane = t & 31;
  const size_t e = size_t(m) * F + size_t(b) * 256 + t;
  const float a = float(gelu_ts(gate[e]) * double(up[e]));
  vals[t] = a;
  if (act_out) act_out[e] = a;
  __syncthreads();
  if (t < 32) {
    float v8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v8[i] = vals[8 * lane + i];
    q8k_block_warp(v8, lane, stage, q8_rec_a(q, m, b), q8_rec_b(q, m, b));
  }
}

// The wide (prefill) form: a warp per 256-block (lane: elements 8L..8L+7),
// eight blocks per CTA and no CTA barrier; same arithmetic, same records as
// hc_geglu_quant_kernel.  Grid (ceil(F / 2048), M).
__global__ void __launch_bounds__(256) hc_geglu_quant_wide_kernel(const float* __restrict__ gate,
                                                               const float* __restrict__ up, int F, Q8Buf q,
                                                               float* __restrict__ act_out) {
  pdl_trigger();
  pdl_wait();
  const int m = int(blockIdx.y), lane = int(threadIdx.x & 31), b = int(blockIdx.x) * 8 + int(threadIdx.x >> 5);
  if (b * 256 >= F) return;
  const size_t e = size_t(m) * F + size_t(b) * 256 + 8 * lane;
  float g[8], u[8], v8[8];
  load8(gate + e, g);
  load8(up + e, u);
#pragma unroll
  for (int i = 0; i < 8; ++i) v8[i] = float(gelu_ts(g[i]) * double(u[i]));
  if (act_out) {
    reinterpret_cast<float4*>(act_out + e)[0] = make_float4(v8[0], v8[1], v8[2], v8[3]);
    reinterpret_cast<float4*>(act_out + e)[1] = make_float4(v8[4], v8[5], v8[6], v8[7]);
  }
  q8k_block_warp(v8, lane, nullptr, q8_rec_a(q, m, b), q8_rec_b(q, m, b));
}

// ---- prefill: many tokens per call -----------------------------------------------------

// QK-norm + RoPE of every token's queries (rounded with the Rust f16 codec,
// lib.rs:590-597) into qh[m][h][256], and, in an own-KV layer, the tokens'
// K (norm + RoPE) and V (unweighted norm) rows into the cache (layers.ts:
// 201-268, 887-911).  One CTA per token, one warp per head vector.
__global__ void hc_prefill_qkv_post_kernel(const float* __restrict__ q, const float* __restrict__ kraw,
                                        const float* __restrict__ vraw, const float* __restrict__ qnw,
                                        const float* __restrict__ knw, const double* __restrict__ cos_t,
                                        const double* __restrict__ sin_t, double eps, int own_kv, float* __restrict__ kc,
                                        float* __restrict__ vc, const int32_t* __restrict__ pos, int H, int KVH, int cap,
                                        float* __restrict__ qh) {
  constexpr int HD = 256;
  const int m = blockIdx.x, lane = threadIdx.x & 31, job = threadIdx.x >> 5;
  const int jobs = own_kv ? H + 2 * KVH : H;
  if (job >= jobs) return;
  float x[8], w[8];
  double c8[8], s8[8];
  load_rope8(cos_t + size_t(m) * (HD / 2), sin_t + size_t(m) * (HD / 2), lane, c8, s8);
  if (job < H) {
    load8(q + (size_t(m) * H + job) * HD + 8 * lane, x);
    load8(qnw + 8 * lane, w);
    head_norm_rope(x, w, true, true, c8, s8, eps, lane);
    float* dst = qh + (size_t(m) * H + job) * HD + 8 * lane;
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = round_f16_rust(x[i]);
    return;
  }
  const int isv = (job - H) / KVH, kvh = (job - H) % KVH;
  load8((isv ? vraw : kraw) + (size_t(m) * KVH + kvh) * HD + 8 * lane, x);
  if (!isv) load8(knw + 8 * lane, w);
  head_norm_rope(x, w, !isv, !isv, c8, s8, eps, lane);
  float* cache = (isv ? vc : kc) + (size_t(pos[m] % cap) * KVH + kvh) * HD + 8 * lane;
  reinterpret_cast<float4*>(cache)[0] = make_float4(x[0], x[1], x[2], x[3]);
  reinterpret_cast<float4*>(cache)[1] = make_float4(x[4], x[5], x[6], x[7]);
}

// Causal GQA attention of PF_QT consecutive tokens x the G query heads of one
// KV head (hp_gqa_attention_f32, lib.rs:539-654, scale 1): KV chunks of
// PF_CK keys are staged with cp.async; each query vector keeps an online
// softmax (running max, f64 exp of the differences, f32 sum) and thread d
// accumulates dimension d of every query's output.  The result is cast with
// the TS f16 codec (castF16Rows, layers.ts:982-988) and its 256-block (one
// head) quantized to Q8_K for the output projection.  Grid
// (ceil(M / PF_QT), KVH); tokens are consecutive positions pos[0] + m.
constexpr int PF_QT = 8, PF_CK = 32;
__global__ void __launch_bounds__(256) hc_prefill_attn_kernel(const float* __restrict__ qh, const float* __restrict__ kc,
                                                          const float* __restrict__ vc, const int32_t* __restrict__ pos,
                                                          int M, int H, int KVH, int cap, Q8Buf qo,
                                                          float* __restrict__ attn_out) {
  constexpr int HD = 256, NQ_MAX = PF_QT * 8;  // G <= 8
  extern __shared__ __align__(16) float psm[];
  const int G = H / KVH, NQ = PF_QT * G, kvh = blockIdx.y, m0 = blockIdx.x * PF_QT;
  float* qs = psm;                          // [NQ][HD]
  float* ks = qs + NQ * HD;                 // [PF_CK][ATT_KSTRIDE]
  float* vs = ks + PF_CK * ATT_KSTRIDE;     // [PF_CK][HD]
  float* ps = vs + PF_CK * HD;              // [NQ][PF_CK]
  __shared__ float alpha[NQ_MAX], run_m[NQ_MAX], run_l[NQ_MAX];
  __shared__ __align__(16) uint8_t stage[8][256];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int mt = min(PF_QT, M - m0);
  // queries: vector qi = token (qi / G) of the tile, head kvh * G + qi % G
  for (int i = tid; i < NQ * HD / 4; i += blockDim.x) {
    const int qi = (4 * i) / HD, d = (4 * i) % HD, mm = min(qi / G, mt - 1);
    reinterpret_cast<float4*>(qs)[i] =
        *reinterpret_cast<const float4*>(qh + (size_t(m0 + mm) * H + kvh * G + qi % G) * HD + d);
  }
  if (tid < NQ) {
    run_m[tid] = -INFINITY;
    run_l[tid] = 0.0f;
  }
  float o[NQ_MAX];
#pragma unroll
  for (int i = 0; i < NQ_MAX; ++i) o[i] = 0.0f;
  const int last = pos[m0 + mt - 1];  // causal: keys 0 .. last
  const int start = max(0, last + 1 - cap);
  for (int k0 = start; k0 <= last; k0 += PF_CK) {
    const int nk = min(PF_CK, last + 1 - k0);
    for (int i = tid; i < PF_CK * (HD / 4); i += blockDim.x) {
      const int j = i / (HD / 4), c = i % (HD / 4), key = k0 + min(j, nk - 1);
      const size_t row = (size_t(key % cap) * KVH + kvh) * HD + 4 * c;
      cp_async16(ks + j * ATT_KSTRIDE + 4 * c, kc + row);
      cp_async16(vs + j * HD + 4 * c, vc + row);
    }
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    // scores, causal per query token
    for (int e = tid; e < NQ * PF_CK; e += blockDim.x) {
      const int qi = e / PF_CK, j = e % PF_CK;
      const float4* qv = reinterpret_cast<const float4*>(qs + qi * HD);
      const float4* kv = reinterpret_cast<const float4*>(ks + j * ATT_KSTRIDE);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 16
      for (int c = 0; c < HD / 4; ++c) {
        const float4 a = qv[c], b = kv[c];
        acc.x = fmaf(a.x, b.x, acc.x);
        acc.y = fmaf(a.y, b.y, acc.y);
        acc.z = fmaf(a.z, b.z, acc.z);
        acc.w = fmaf(a.w, b.w, acc.w);
      }
      const int mq = qi / G;
      const bool ok = j < nk && mq < mt && k0 + j <= pos[m0 + mq];
      ps[e] = ok ? (acc.x + acc.y) + (acc.z + acc.w) : -INFINITY;
    }
    __syncthreads();
    // online softmax: warp per query vector, lane = key
    for (int qi = warp; qi < NQ; qi += 8) {
      const float sc = ps[qi * PF_CK + lane];
      float mx = sc;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mo = run_m[qi], mn = fmaxf(mo, mx);
      const float p = (sc == -INFINITY) ? 0.0f : float(exp(double(sc - mn)));
      float sum = p;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      ps[qi * PF_CK + lane] = p;
      __syncwarp();
      if (lane == 0) {
        const float a = (mo == -INFINITY) ? 0.0f : float(exp(double(mo - mn)));
        alpha[qi] = a;
        run_l[qi] = run_l[qi] * a + sum;
        run_m[qi] = mn;
      }
    }
    __syncthreads();
    // outputs: thread d owns dimension d of every query vector
    const int d = tid;
#pragma unroll
    for (int qi = 0; qi < NQ_MAX; ++qi) {
      if (qi < NQ) {
        float acc = o[qi] * alpha[qi];
        const float* pr = ps + qi * PF_CK;
        for (int j = 0; j < nk; ++j) acc += pr[j] * vs[j * HD + d];
        o[qi] = acc;
      }
    }
    __syncthreads();
  }
  // normalize, f16 cast, quantize each (token, head) block
  float* outv = ks;  // reuse: [NQ][HD]
#pragma unroll
  for (int qi = 0; qi < NQ_MAX; ++qi)
    if (qi < NQ) outv[qi * HD + tid] = round_f16_ts(float(double(o[qi]) / double(run_l[qi])));
  __syncthreads();
  for (int qi = warp; qi < NQ; qi += 8) {
    const int mq = qi / G, h = kvh * G + qi % G;
    if (mq >= mt) continue;
    float v8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v8[i] = outv[qi * HD + 8 * lane + i];
    if (attn_out) {
      float* dst = attn_out + (size_t(m0 + mq) * H + h) * HD + 8 * lane;
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[i] = v8[i];
    }
    q8k_block_warp(v8, lane, stage[warp], q8_rec_a(qo, m0 + mq, h), q8_rec_b(qo, m0 + mq, h));
  }
}

// Split form of the prefill attention: the keys of a query tile are cut into
// PF_SK-key splits, one CTA per (tile, split, KV head), so the causal work of
// the long tiles spreads over many CTAs; hc_prefill_attn_merge_kernel merges
// the splits.  Per CTA: the PF_QT tokens x G heads of the tile (qs, rows
// padded for conflict-free reads), keys in PF_CK chunks (online softmax:
// running max, f64 exp of the differences, f32 sums), scores as 2 x 2
// register blocks (a warp covers 8 query vectors x 16 keys), outputs with
// thread d = dimension over 4 keys per step.  Writes the split's max, sum and
// unnormalized output per (token, head) to part_m / part_l / part_o at
// ((token * H + head) * nsplit + split).
constexpr int PF_SK = 128;       // keys per split
constexpr int PF_QSTRIDE = 260;  // floats per staged query row
__global__ void __launch_bounds__(256) hc_prefill_attn_split_kernel(const float* __restrict__ qh,
                                                                const float* __restrict__ kc,
                                                                const float* __restrict__ vc,
                                                                const int32_t* __restrict__ pos, int M, int H, int KVH,
                                                                int cap, int nsplit, float* __restrict__ part_m,
                                                                float* __restrict__ part_l, float* __restrict__ part_o) {
  constexpr int HD = 256, NQ_MAX = PF_QT * 4;  // G <= 4
  extern __shared__ __align__(16) float psm[];
  const int G = H / KVH, NQ = PF_QT * G, kvh = int(blockIdx.y);
  const int tile = int(blockIdx.x) / nsplit, split = int(blockIdx.x) % nsplit, m0 = tile * PF_QT;
  const int mt = min(PF_QT, M - m0);
  const int last = pos[m0 + mt - 1];
  const int start = max(0, last + 1 - cap);
  const int k_lo = start + split * PF_SK, k_hi = min(start + (split + 1) * PF_SK, last + 1);
  if (k_lo >= k_hi) return;  // this tile's window ends before the split
  float* qs = psm;                           // [NQ][PF_QSTRIDE]
  float* ks = qs + NQ * PF_QSTRIDE;          // [PF_CK][ATT_KSTRIDE]
  float* vs = ks + PF_CK * ATT_KSTRIDE;      // [PF_CK][HD]
  float* ps = vs + PF_CK * HD;               // [NQ][PF_CK]
  __shared__ float alpha[NQ_MAX], run_m[NQ_MAX], run_l[NQ_MAX];
  const int tid = int(threadIdx.x), lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < NQ * HD / 4; i += int(blockDim.x)) {
    const int qi = (4 * i) / HD, d = (4 * i) % HD, mm = min(qi / G, mt - 1);
    *reinterpret_cast<float4*>(qs + qi * PF_QSTRIDE + d) =
        *reinterpret_cast<const float4*>(qh + (size_t(m0 + mm) * H + kvh * G + qi % G) * HD + d);
  }
  if (tid < NQ) {
    run_m[tid] = -INFINITY;
    run_l[tid] = 0.0f;
  }
  float o[NQ_MAX];
#pragma unroll
  for (int i = 0; i < NQ_MAX; ++i) o[i] = 0.0f;
  for (int k0 = k_lo; k0 < k_hi; k0 += PF_CK) {
    const int nk = min(PF_CK, k_hi - k0);
    for (int i = tid; i < PF_CK * (HD / 4); i += int(blockDim.x)) {
      const int j = i / (HD / 4), c = i % (HD / 4), key = k0 + min(j, nk - 1);
      const size_t row = (size_t(key % cap) * KVH + kvh) * HD + 4 * c;
      cp_async16(ks + j * ATT_KSTRIDE + 4 * c, kc + row);
      cp_async16(vs + j * HD + 4 * c, vc + row);
    }
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    // scores: warp w covers query pairs 4 (w % 4) .. + 3 and key pairs
    // 8 (w / 4) .. + 7 (lane: query pair lane / 8, key pair lane % 8); more
    // query vectors than 32 take further passes
    for (int qb = 0; qb < NQ; qb += 32) {
      const int qa = qb + 2 * (4 * (warp & 3) + (lane >> 3)), kb = 2 * (8 * (warp >> 2) + (lane & 7));
      if (qa < NQ) {
        const float4* q0 = reinterpret_cast<const float4*>(qs + qa * PF_QSTRIDE);
        const float4* q1 = reinterpret_cast<const float4*>(qs + (qa + 1) * PF_QSTRIDE);
        const float4* kv0 = reinterpret_cast<const float4*>(ks + kb * ATT_KSTRIDE);
        const float4* kv1 = reinterpret_cast<const float4*>(ks + (kb + 1) * ATT_KSTRIDE);
        float4 a00 = make_float4(0.f, 0.f, 0.f, 0.f), a01 = a00, a10 = a00, a11 = a00;
#pragma unroll 8
        for (int c = 0; c < HD / 4; ++c) {
          const float4 x0 = q0[c], x1 = q1[c], y0 = kv0[c], y1 = kv1[c];
          a00.x = fmaf(x0.x, y0.x, a00.x); a00.y = fmaf(x0.y, y0.y, a00.y);
          a00.z = fmaf(x0.z, y0.z, a00.z); a00.w = fmaf(x0.w, y0.w, a00.w);
          a01.x = fmaf(x0.x, y1.x, a01.x); a01.y = fmaf(x0.y, y1.y, a01.y);
          a01.z = fmaf(x0.z, y1.z, a01.z); a01.w = fmaf(x0.w, y1.w, a01.w);
          a10.x = fmaf(x1.x, y0.x, a10.x); a10.y = fmaf(x1.y, y0.y, a10.y);
          a10.z = fmaf(x1.z, y0.z, a10.z); a10.w = fmaf(x1.w, y0.w, a10.w);
          a11.x = fmaf(x1.x, y1.x, a11.x); a11.y = fmaf(x1.y, y1.y, a11.y);
          a11.z = fmaf(x1.z, y1.z, a11.z); a11.w = fmaf(x1.w, y1.w, a11.w);
        }
        const float4 acc[2][2] = {{a00, a01}, {a10, a11}};
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int qi = qa + i, key = kb + j;
            const int mq = qi / G;
            const bool ok = key < nk && mq < mt && k0 + key <= pos[m0 + min(mq, mt - 1)];
            const float4 v = acc[i][j];
            ps[qi * PF_CK + key] = ok ? (v.x + v.y) + (v.z + v.w) : -INFINITY;
          }
      }
    }
    __syncthreads();
    // online softmax: warp per query vector, lane = key
    for (int qi = warp; qi < NQ; qi += 8) {
      const float sc = ps[qi * PF_CK + lane];
      float mx = sc;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mo = run_m[qi], mn = fmaxf(mo, mx);
      const float p = (sc == -INFINITY) ? 0.0f : float(exp(double(sc - mn)));
      float sum = p;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      ps[qi * PF_CK + lane] = p;
      __syncwarp();
      if (lane == 0) {
        const float a = (mo == -INFINITY) ? 0.0f : float(exp(double(mo - mn)));
        alpha[qi] = a;
        run_l[qi] = run_l[qi] * a + sum;
        run_m[qi] = mn;
      }
    }
    __syncthreads();
    // outputs: thread d owns dimension d of every query vector, 4 keys per step
    const int d = tid;
#pragma unroll
    for (int qi = 0; qi < NQ_MAX; ++qi)
      if (qi < NQ) o[qi] *= alpha[qi];
    for (int j = 0; j < nk; j += 4) {
      const float b0 = vs[j * HD + d], b1 = vs[(j + 1) * HD + d], b2 = vs[(j + 2) * HD + d],
                  b3 = vs[(j + 3) * HD + d];
#pragma unroll
      for (int qi = 0; qi < NQ_MAX; ++qi) {
        if (qi < NQ) {
          const float4 pr = *reinterpret_cast<const float4*>(ps + qi * PF_CK + j);
          o[qi] += pr.x * b0 + pr.y * b1 + pr.z * b2 + pr.w * b3;
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int qi = 0; qi < NQ_MAX; ++qi) {
    if (qi < NQ && qi / G < mt) {
      const size_t ix = (size_t(m0 + qi / G) * H + kvh * G + qi % G) * nsplit + split;
      if (tid == 0) {
        part_m[ix] = run_m[qi];
        part_l[ix] = run_l[qi];
      }
      part_o[ix * HD + tid] = o[qi];
    }
  }
}

// Merges the splits of one (token, head): the splits of its tile's window
// that reach the token (global max, f64-exp weights, f64 sum, weighted
// outputs), the TS f16 cast (castF16Rows) and the head's Q8_K block for the
// output projection.  Grid (M, H), thread d = dimension.
__global__ void __launch_bounds__(256) hc_prefill_attn_merge_kernel(const float* __restrict__ part_m,
                                                                const float* __restrict__ part_l,
                                                                const float* __restrict__ part_o,
                                                                const int32_t* __restrict__ pos, int M, int H, int cap,
                                                                int nsplit, Q8Buf qo, float* __restrict__ attn_out) {
  constexpr int HD = 256;
  __shared__ float w[64];
  __shared__ double lsum;
  __shared__ float vec[HD];
  const int m = int(blockIdx.x), h = int(blockIdx.y), d = int(threadIdx.x);
  const int tile = m / PF_QT, mt = min(PF_QT, M - tile * PF_QT);
  const int last = pos[tile * PF_QT + mt - 1];
  const int start = max(0, last + 1 - cap);
  const int ns = min(nsplit, (pos[m] - start) / PF_SK + 1);  // splits holding keys <= pos[m]
  const size_t base = (size_t(m) * H + h) * nsplit;
  if (d == 0) {
    float mx = -INFINITY;
    for (int s = 0; s < ns; ++s) mx = fmaxf(mx, part_m[base + s]);
    double l = 0.0;
    for (int s = 0; s < ns; ++s) {
      const float ms = part_m[base + s];
      const float ws = ms == -INFINITY ? 0.0f : float(exp(double(ms - mx)));
      w[s] = ws;
      l += double(ws) * double(part_l[base + s]);
    }
    lsum = l;
  }
  __syncthreads();
  float o = 0.0f;
  for (int s = 0; s < ns; ++s) o += w[s] * part_o[(base + s) * HD + d];
  const float n = round_f16_ts(float(double(o) / lsum));
  vec[d] = n;
  if (attn_out) attn_out[(size_t(m) * H + h) * HD + d] = n;
  __syncthreads();
  if (d < 32) {
    float v8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v8[i] = vec[8 * d + i];
    q8k_block_warp(v8, d, nullptr, q8_rec_a(qo, m, h), q8_rec_b(qo, m, h));
  }
}

// ---- launch helpers ---------------------------------------------------------------------

template <typename... KArgs, typename... Args>
static cudaError_t pdl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

cudaError_t launch_rope_gather(const int32_t* pos, int M, int half, const double* cos_tab, const double* sin_tab,
                               int table_rows, double theta_scale, double* cos_t, double* sin_t, cudaStream_t st) {
  if (half > 512) return cudaErrorInvalidValue;
  return pdl_launch(hc_rope_gather_kernel, dim3(M), dim3(128), 0, st, pos, half, cos_tab, sin_tab, table_rows,
                    theta_scale, cos_t, sin_t);
}

cudaError_t launch_embed(const uint8_t* w, int type, int nb, int vocab, const int32_t* ids, float* hidden, int M, int D,
                         double scale, int* err, cudaStream_t st) {
  return pdl_launch(hc_embed_kernel, dim3(M), dim3(256), 0, st, w, type, nb, vocab, ids, hidden, D, scale, err);
}

cudaError_t launch_norm_quant(bool resid, const float* x, float* x_out, const float* y, const float* w_post,
                              const float* w_pre, double eps, int M, int D, const Q8Buf& q, float* n_out,
                              cudaStream_t st) {
  const dim3 grid(M), block(D / 8);
  if (resid)
    return pdl_launch(hc_norm_quant_kernel<true>, grid, block, 0, st, x, x_out, y, w_post, w_pre, eps, D, q, n_out);
  return pdl_launch(hc_norm_quant_kernel<false>, grid, block, 0, st, x, x_out, y, w_post, w_pre, eps, D, q, n_out);
}

size_t attn_smem_bytes(int M, int H, int KVH) {
  const int NQ = M * (H / KVH);
  return sizeof(float) * (size_t(ATT_CHUNK) * ATT_KSTRIDE * 2 + size_t(NQ) * 256 + size_t(NQ) * ATT_CHUNK);
}

namespace {
using AttnKernel = decltype(&hc_attn_partial_kernel<false>);
// Wide forms sized to NQ = 8, 12, ..., 32 query vectors per KV head (four
// heads per KV head at 2..8 tokens): ceil(NQ / 8) score slots and
// ceil(NQ / 2) output slots per half: every output slot holds a query, the
// two halves each take one output pass, and a score lane idles at most one
// slot (at NQ = 20, lanes 4..7 have two queries for three slots).  Index
// (NQ - 8) / 4.
constexpr AttnKernel kAttnSized[] = {
    hc_attn_partial_kernel<true, 1, 4>,  hc_attn_partial_kernel<true, 2, 6>,  hc_attn_partial_kernel<true, 2, 8>,
    hc_attn_partial_kernel<true, 3, 10>, hc_attn_partial_kernel<true, 3, 12>, hc_attn_partial_kernel<true, 4, 14>,
    hc_attn_partial_kernel<true, 4, 16>};

AttnKernel attn_wide_kernel(int nq) {
  if (nq >= 8 && nq <= 32 && nq % 4 == 0) return kAttnSized[(nq - 8) / 4];
  return hc_attn_partial_kernel<true>;
}
}  // namespace

cudaError_t launch_attention(const float* q, const float* kraw, const float* vraw, const float* qnw, const float* knw,
                             const double* cos_t, const double* sin_t, double eps, bool own_kv, float* kc, float* vc,
                             const int32_t* pos, int M, int H, int KVH, int cap, float scale, float* part_m,
                             float* part_l, float* part_o, int* err, cudaStream_t st) {
  if (cap % ATT_CHUNK != 0 || cap > 4096) return cudaErrorInvalidValue;
  const size_t smem = attn_smem_bytes(M, H, KVH);
  if (smem > ATT_MAX_SMEM) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr{0};
  const cudaError_t ea = once_per_current_device(attr, [] {
    const AttnKernel all[] = {hc_attn_partial_kernel<false>, hc_attn_partial_kernel<true>, kAttnSized[0], kAttnSized[1],
                              kAttnSized[2],              kAttnSized[3],             kAttnSized[4], kAttnSized[5],
                              kAttnSized[6]};
    for (AttnKernel k : all) {
      const void* fn = reinterpret_cast<const void*>(k);
      const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(ATT_MAX_SMEM));
      if (e != cudaSuccess) return e;
      // maximal shared-memory carveout: the SMs still running the QKV GEMV's
      // CTAs can take an attention CTA (~140 KB) without draining first
      // (measured: decode +1.6%; the GEMVs keep the default split)
      use_max_carveout(fn);
    }
    return cudaSuccess;
  });
  if (ea != cudaSuccess) return ea;
  const int chunks = cap / ATT_CHUNK;
  // more than four query vectors per KV head: the register-blocked form
  if (M * (H / KVH) > ATT_THREADS / ATT_CHUNK)
    return pdl_launch(attn_wide_kernel(M * (H / KVH)), dim3(chunks, KVH), dim3(ATT_WIDE_THREADS), smem, st, q, kraw, vraw, qnw,
                      knw, cos_t, sin_t, eps, int(own_kv), kc, vc, pos, M, H, KVH, cap, scale, part_m, part_l, part_o,
                      err);
  return pdl_launch(hc_attn_partial_kernel<false>, dim3(chunks, KVH), dim3(ATT_THREADS), smem, st, q, kraw, vraw, qnw,
                    knw, cos_t, sin_t, eps, int(own_kv), kc, vc, pos, M, H, KVH, cap, scale, part_m, part_l, part_o,
                    err);
}

cudaError_t launch_attn_combine(const float* part_m, const float* part_l, const float* part_o, const int32_t* pos,
                                int M, int H, int KVH, int cap, const Q8Buf& q, float* attn_out, cudaStream_t st) {
  return pdl_launch(hc_attn_combine_kernel, dim3(M, H), dim3(256), 0, st, part_m, part_l, part_o, pos, M, H, KVH, cap, q,
                    attn_out);
}

cudaError_t launch_geglu_quant(const float* gate, const float* up, int M, int F, const Q8Buf& q, float* act_out,
                               cudaStream_t st) {
  if (M >= GEGLU_WIDE_MIN_COLS)
    return pdl_launch(hc_geglu_quant_wide_kernel, dim3((F / 256 + 7) / 8, M), dim3(256), 0, st, gate, up, F, q,
                      act_out);
  return pdl_launch(hc_geglu_quant_kernel, dim3(F / 256, M), dim3(256), 0, st, gate, up, F, q, act_out);
}

cudaError_t launch_prefill_qkv_post(const float* q, const float* kraw, const float* vraw, const float* qnw,
                                   const float* knw, const double* cos_t, const double* sin_t, double eps, bool own_kv,
                                   float* kc, float* vc, const int32_t* pos, int M, int H, int KVH, int cap, float* qh,
                                   cudaStream_t st) {
  const int jobs = own_kv ? H + 2 * KVH : H;
  if (jobs > 32) return cudaErrorInvalidValue;
  hc_prefill_qkv_post_kernel<<<M, 32 * jobs, 0, st>>>(q, kraw, vraw, qnw, knw, cos_t, sin_t, eps, int(own_kv), kc, vc, pos,
                                                   H, KVH, cap, qh);
  return cudaGetLastError();
}

size_t prefill_attn_smem_bytes(int H, int KVH) {
  const int NQ = PF_QT * (H / KVH);
  return sizeof(float) * (size_t(NQ) * 256 + size_t(PF_CK) * ATT_KSTRIDE + size_t(PF_CK) * 256 + size_t(NQ) * PF_CK);
}

size_t prefill_split_smem_bytes(int H, int KVH) {
  const int NQ = PF_QT * (H / KVH);
  return sizeof(float) * (size_t(NQ) * PF_QSTRIDE + size_t(PF_CK) * ATT_KSTRIDE + size_t(PF_CK) * 256 +
                          size_t(NQ) * PF_CK);
}

int prefill_attn_splits(int cap, int max_pos) {
  const int window = min(cap, max_pos + 1);
  return (window + PF_SK - 1) / PF_SK;
}

cudaError_t launch_prefill_attention_split(const float* qh, const float* kc, const float* vc, const int32_t* pos,
                                           int M, int H, int KVH, int cap, int nsplit, float* part_m, float* part_l,
                                           float* part_o, const Q8Buf& qo, float* attn_out, cudaStream_t st) {
  if (H / KVH > 4 || nsplit < 1 || nsplit > 64) return cudaErrorInvalidValue;
  const size_t smem = prefill_split_smem_bytes(H, KVH);
  static std::atomic<uint64_t> attr{0};
  const cudaError_t ea = once_per_current_device(attr, [] {
    return cudaFuncSetAttribute(hc_prefill_attn_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  if (ea != cudaSuccess) return ea;
  const int tiles = (M + PF_QT - 1) / PF_QT;
  hc_prefill_attn_split_kernel<<<dim3(unsigned(tiles * nsplit), unsigned(KVH)), 256, smem, st>>>(
      qh, kc, vc, pos, M, H, KVH, cap, nsplit, part_m, part_l, part_o);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  hc_prefill_attn_merge_kernel<<<dim3(unsigned(M), unsigned(H)), 256, 0, st>>>(part_m, part_l, part_o, pos, M, H, cap,
                                                                           nsplit, qo, attn_out);
  return cudaGetLastError();
}

cudaError_t launch_prefill_attention(const float* qh, const float* kc, const float* vc, const int32_t* pos, int M,
                                     int H, int KVH, int cap, const Q8Buf& qo, float* attn_out, cudaStream_t st) {
  if (H / KVH > 8) return cudaErrorInvalidValue;
  const size_t smem = prefill_attn_smem_bytes(H, KVH);
  // the limit is set once per device, so it is the bound of the widest group
  // this kernel accepts (8 query heads per KV head), not this call's need
  static std::atomic<uint64_t> attr{0};
  const cudaError_t ea = once_per_current_device(attr, [] {
    return cudaFuncSetAttribute(hc_prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(prefill_attn_smem_bytes(8, 1)));
  });
  if (ea != cudaSuccess) return ea;
  hc_prefill_attn_kernel<<<dim3(unsigned((M + PF_QT - 1) / PF_QT), unsigned(KVH)), 256, smem, st>>>(
      qh, kc, vc, pos, M, H, KVH, cap, qo, attn_out);
  return cudaGetLastError();
}

}  // namespace hc
