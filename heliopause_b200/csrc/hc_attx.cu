// hc_attx.cu -- decode / verify attention in the reference's exact f32 order.
//
// hp_gqa_attention_f32 (lib.rs:539-654), as the WASM provider calls it per
// layer (layers.ts:304-334: query rounded to f16 with the Rust codec, scale
// 1, causal mask, value layout [dim][head][slot]), computes for every
// (token, query head):
//   dot_j   = sequential f32 sum over i of fround(q_i * k_j,i)
//   score_j = fround(dot_j * scale) + mask_j            (-inf where masked)
//   p_j     = f32(exp(f64(score_j - max)))              (0 where masked)
//   sum     = sequential f32 sum over j of p_j
//   out_d   = sequential f32 sum over j of fround(fround(p_j / sum) * v_j,d)
// over the keys j = 0 .. count-1 in order (count = min(capacity, top + 1),
// key j at slot (start + j) % capacity).  The kernels below reproduce every
// one of those roundings in that order, so the output equals the
// reference's bit for bit (given bit-equal inputs); only independent chains
// run in parallel:
//   hc_attx_scores_kernel  grid (64-slot chunks, KV heads): the QK-norm,
//                          RoPE and f16 rounding of the queries, this step's
//                          K/V rows (written to the cache), one sequential
//                          256-term dot per (query, key);
//   hc_attx_softmax_kernel grid (tokens x heads): the max, the f64 exps, the
//                          4096-term sequential sum (evaluated as integer
//                          runs inside binades, the same f32 value), the
//                          divisions;
//   hc_attx_pv_kernel      grid (KV head x 32-dim slice, groups of 1-4 query
//                          vectors): one sequential chain per (query, dim)
//                          over all keys, lane = dim, then the TS f16 cast of
//                          the output (castF16Rows, layers.ts:982-988).  A
//                          producer warp feeds a ring of 256-key stages: the
//                          stage's V slice [256 slots][32 dims] as one 2-D
//                          TMA tensor copy
//                          (per-key bulk copies where the stage wraps the
//                          slot ring) and the group's probabilities as one
//                          bulk copy per query, completion on the stage's
//                          mbarrier; the chain warps do nothing but the
//                          chain, whose dependent adds bound the kernel.
// The Q8_K quantization of the cast output for the O projection follows as
// its own launch.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <mutex>

#include "hc_bulk.cuh"
#include "hc_common.cuh"
#include "hc_decmath.cuh"
#include "hc_decode.cuh"
#include "hc_kernels.cuh"

namespace hc {

namespace {

constexpr int AX_CH = 64;            // key slots per scores CTA
constexpr int AX_KSTRIDE = 256 + 4;  // floats per staged K row (conflict-free 16-byte reads)
constexpr int AX_QL = 4;             // query lanes of the scores CTA (256 threads / 64 keys)
constexpr int AX_SM_THREADS = 1024;  // softmax CTA
constexpr int AX_PV_CW_MAX = 4;      // chain warps per PV CTA, at most
constexpr int AX_PV_TC = 256;        // keys per ring stage
constexpr int AX_PV_NS = 4;          // ring stages (three stages of copies ahead of the chain)
constexpr int AX_PV_DS = 32;         // dims per CTA: one per lane
// floats per stage: V [TC][32], probabilities [QG][TC]
__host__ __device__ constexpr int pv_stage_floats(int qg) { return AX_PV_TC * AX_PV_DS + qg * AX_PV_TC; }

struct KeyRange {
  int count, start, maxpos;
};

__device__ __forceinline__ KeyRange key_range(const int32_t* pos, int M, int cap) {
  int mx = 0;
  for (int i = 0; i < M; ++i) mx = max(mx, pos[i]);
  KeyRange r;
  r.maxpos = mx;
  r.count = min(cap, mx + 1);
  r.start = mx + 1 - r.count;
  return r;
}

// U query chains of one key (queries q0, q0 + 4, ...): each dot is the
// reference's sequential chain over the 256 dims; the key row's 16-byte
// pieces are read once for all U.
template <int U>
__device__ __forceinline__ void score_chains(const float4* __restrict__ kv, const float* __restrict__ qs, int q0,
                                             bool key, int kpos, int j, int G, int H, int kvh, int cap, float scale,
                                             const int32_t* __restrict__ pos, float* __restrict__ scores) {
  float dot[U];
#pragma unroll
  for (int u = 0; u < U; ++u) dot[u] = 0.0f;
#pragma unroll 4
  for (int i4 = 0; i4 < 64; ++i4) {
    const float4 b = kv[i4];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float4 a = reinterpret_cast<const float4*>(qs + (q0 + AX_QL * u) * 256)[i4];
      dot[u] = __fadd_rn(dot[u], __fmul_rn(a.x, b.x));
      dot[u] = __fadd_rn(dot[u], __fmul_rn(a.y, b.y));
      dot[u] = __fadd_rn(dot[u], __fmul_rn(a.z, b.z));
      dot[u] = __fadd_rn(dot[u], __fmul_rn(a.w, b.w));
    }
  }
  if (!key) return;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int qi = q0 + AX_QL * u, m = qi / G, h = kvh * G + qi % G;
    // mask 0 where the key is visible: fround(fround(dot * scale) + 0)
    scores[(size_t(m) * H + h) * cap + j] = kpos <= pos[m] ? __fadd_rn(__fmul_rn(dot[u], scale), 0.0f) : -INFINITY;
  }
}

__global__ void __launch_bounds__(256) hc_attx_scores_kernel(
    const float* __restrict__ q, const float* __restrict__ kraw, const float* __restrict__ vraw,
    const float* __restrict__ qnw, const float* __restrict__ knw, const double* __restrict__ cos_t,
    const double* __restrict__ sin_t, double eps, int own_kv, float* __restrict__ kc, float* __restrict__ vc,
    const int32_t* __restrict__ pos, int M, int H, int KVH, int cap, float scale, float* __restrict__ scores) {
  constexpr int HD = 256;
  extern __shared__ __align__(16) float sm[];
  const int chunk = int(blockIdx.x), kvh = int(blockIdx.y);
  const int G = H / KVH, NQ = M * G;
  float* ks = sm;                      // [AX_CH][AX_KSTRIDE]
  float* qs = ks + AX_CH * AX_KSTRIDE; // [NQ][HD]
  pdl_trigger();
  const KeyRange kr = key_range(pos, M, cap);  // pos is set before the step starts
  const int t0 = chunk * AX_CH;
  // a slot s holds key j = (s - start) mod cap when j < count
  // every slot holds a key once the ring is full; before that start = 0 and
  // the keys are the slots below count
  const bool any = kr.count == cap || t0 < kr.count;
  bool fresh = false;
  for (int i = 0; i < M; ++i) {
    const int s = pos[i] % cap;
    fresh |= (s >= t0 && s < t0 + AX_CH);
  }
  if (!any) {
    pdl_wait();
    return;
  }
  {  // the chunk's K rows, before the wait (rows this step writes are replaced below)
    constexpr int PIECES = HD * 4 / 16;
    const int nw = int(blockDim.x >> 5), cw0 = NQ < nw ? NQ : 0;  // query warps issue no copies
    const int ncp = (nw - cw0) * 32;
    if (int(threadIdx.x >> 5) >= cw0)
      for (int i = int(threadIdx.x) - cw0 * 32; i < AX_CH * PIECES; i += ncp) {
        const int t = i / PIECES, c = i % PIECES;
        cp_async16(ks + t * AX_KSTRIDE + 4 * c, kc + (size_t(t0 + t) * KVH + kvh) * HD + 4 * c);
      }
    cp_async_commit();
    // the same slots' V rows (every KV head) into L2 for the p.v kernel two
    // launches later, which streams them in key order
    if (kvh == 0 && threadIdx.x < 8) {
      const char* vrow = reinterpret_cast<const char*>(vc + size_t(t0) * KVH * HD);
      const uint32_t span = uint32_t(AX_CH / 8) * uint32_t(KVH) * HD * 4;  // 8 pieces of the 64 slots
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(vrow + size_t(threadIdx.x) * span), "r"(span)
                   : "memory");
    }
  }
  const int lane = int(threadIdx.x) & 31, warp = int(threadIdx.x) >> 5, warps = int(blockDim.x) >> 5;
  float qw[8], kw[8];
  load8(qnw + 8 * lane, qw);
  if (own_kv && fresh) load8(knw + 8 * lane, kw);
  pdl_wait();
  // queries: QK-norm + RoPE, then the Rust f16 codec (lib.rs:590-597)
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
  __syncthreads();
  // this step's K/V rows: own-KV layers compute them (K: norm + RoPE, V:
  // unweighted norm; layers.ts:241-268) and write the cache (layers.ts:887-911);
  // shared-KV layers read the source layer's rows from the cache
  if (fresh) {
    for (int job = warp; job < 2 * M; job += warps) {
      const int m = job >> 1, isv = job & 1, p = pos[m], s = p % cap;
      if (s < t0 || s >= t0 + AX_CH) continue;
      float* cache = (isv ? vc : kc) + (size_t(s) * KVH + kvh) * HD + 8 * lane;
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
      if (!isv) {
        float* staged = ks + (s - t0) * AX_KSTRIDE + 8 * lane;
#pragma unroll
        for (int i = 0; i < 8; ++i) staged[i] = x[i];
      }
    }
  }
  __syncthreads();
  // scores: thread (key t = tid % 64, query lane ql = tid / 64) walks queries
  // ql, ql + 4, ...; each dot is the reference's sequential chain
  const int t = int(threadIdx.x) % AX_CH, ql = int(threadIdx.x) / AX_CH;
  const int j = (t0 + t - kr.start + cap) % cap;
  const bool key = j < kr.count;
  const int kpos = kr.start + j;  // absolute position of the key
  const float4* kv = reinterpret_cast<const float4*>(ks + t * AX_KSTRIDE);
  // this thread's queries ql, ql + 4, ...: passes of at most 4 chains, each
  // pass sized to the chains it really has
  const int mine = NQ > ql ? (NQ - ql + AX_QL - 1) / AX_QL : 0;
  for (int u0 = 0; u0 < mine; u0 += 4) {
    const int cnt = min(4, mine - u0), q0 = ql + AX_QL * u0;
    switch (cnt) {
      case 1: score_chains<1>(kv, qs, q0, key, kpos, j, G, H, kvh, cap, scale, pos, scores); break;
      case 2: score_chains<2>(kv, qs, q0, key, kpos, j, G, H, kvh, cap, scale, pos, scores); break;
      case 3: score_chains<3>(kv, qs, q0, key, kpos, j, G, H, kvh, cap, scale, pos, scores); break;
      default: score_chains<4>(kv, qs, q0, key, kpos, j, G, H, kvh, cap, scale, pos, scores); break;
    }
  }
}

// The sequential f32 sum of the probabilities (lib.rs:627-635), computed in
// parallel with the same result.  While the running sum stays inside one
// binade [2^e, 2^(e+1)) every partial sum is a multiple of u = 2^(e-23), so
// fl(s + x) = s + u*k with k = x/u rounded to the nearest integer (x >= 0,
// no tie): the adds of a run inside one binade are integer adds and may be
// regrouped.  (Below 2^-125 the grid is 2^-149 and every add is exact: binade
// index -126.)  An f64 prefix sum P locates the partial sums: the sum only
// grows, so after j + 1 terms |s_j - P_j| <= (j + 1) 2^-24 s_j, and s_j is at
// least the largest term so far.  A key whose bracket
// [max(P_{j-1}(1 - m), max_{i<j} x_i), P_j (1 + m)], m = (j + 2) 2^-23, lies in
// one binade and whose x/u is not a tie is "safe": its add is u*k.  The
// others (key 0, binade crossings, ties, brackets that touch a boundary) are
// added in key order by one thread, each followed by the integer total of
// the safe run after it, which is the partial sum the dependent chain
// reaches at the run's end.
constexpr int AX_SM_KPT = 4;      // keys per thread: 4 x 1024 covers the 4096-slot cap
constexpr int AX_SM_LIST = 1024;  // unsafe keys held; more take the plain chain
static_assert(AX_SM_KPT * AX_SM_THREADS == 4096, "one pass over the largest key count");

__device__ __forceinline__ int binade_index(double v) {  // v >= 0
  const int e = int((__double_as_longlong(v) >> 52) & 0x7ff) - 1023;
  return v > 0.0 ? max(e, -126) : -126;
}

__global__ void __launch_bounds__(AX_SM_THREADS) hc_attx_softmax_kernel(const float* __restrict__ scores,
                                                                        const int32_t* __restrict__ pos, int M, int H,
                                                                        int cap, float* __restrict__ rprob) {
  __shared__ __align__(16) float ps[4096];
  __shared__ signed char eb[4096];           // binade index of each key's bracket
  __shared__ int uq[AX_SM_LIST];             // unsafe keys, in order
  __shared__ unsigned uk[AX_SM_LIST + 1];    // sum of the safe k before each unsafe key (+ the total)
  __shared__ __align__(8) float2 xr[AX_SM_LIST];  // per unsafe key: its term, the run after it
  __shared__ double dsum[32];
  __shared__ float fmx[32], fpm[32];
  __shared__ int nsum[32];
  __shared__ unsigned ksum[32];
  __shared__ int s_nuns;
  __shared__ float s_sum;
  const int m = int(blockIdx.x) / H, h = int(blockIdx.x) % H;
  const int t = int(threadIdx.x), lane = t & 31, w = t >> 5;
  pdl_trigger();
  const KeyRange kr = key_range(pos, M, cap);
  pdl_wait();
  const float* sc = scores + (size_t(m) * H + h) * cap;
  const int j0 = AX_SM_KPT * t;
  float x[AX_SM_KPT];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < AX_SM_KPT; ++i) {
    x[i] = j0 + i < kr.count ? sc[j0 + i] : -INFINITY;
    mx = fmaxf(mx, x[i]);
  }
  // the max over every key (exact and order-free; every token sees its own key)
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) fmx[w] = mx;
  __syncthreads();
  mx = fmx[lane];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  // the terms, their f64 prefix sums and running maxima
  double c[AX_SM_KPT];
  double run = 0.0;
  float pmax = 0.0f;
#pragma unroll
  for (int i = 0; i < AX_SM_KPT; ++i) {
    x[i] = x[i] == -INFINITY ? 0.0f : float(exp(double(__fsub_rn(x[i], mx))));
    run += double(x[i]);
    c[i] = run;
    pmax = fmaxf(pmax, x[i]);
  }
  reinterpret_cast<float4*>(ps)[t] = make_float4(x[0], x[1], x[2], x[3]);
  double incl = run;
  float pm = pmax;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const double v = __shfl_up_sync(0xffffffffu, incl, off);
    const float q = __shfl_up_sync(0xffffffffu, pm, off);
    if (lane >= off) {
      incl += v;
      pm = fmaxf(pm, q);
    }
  }
  if (lane == 31) {
    dsum[w] = incl;
    fpm[w] = pm;
  }
  double excl = __shfl_up_sync(0xffffffffu, incl, 1);
  float pex = __shfl_up_sync(0xffffffffu, pm, 1);
  if (lane == 0) {
    excl = 0.0;
    pex = 0.0f;
  }
  __syncthreads();
  if (w == 0) {
    const double v = dsum[lane];
    const float q = fpm[lane];
    double iv = v;
    float iq = q;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const double a = __shfl_up_sync(0xffffffffu, iv, off);
      const float b = __shfl_up_sync(0xffffffffu, iq, off);
      if (lane >= off) {
        iv += a;
        iq = fmaxf(iq, b);
      }
    }
    double ev = __shfl_up_sync(0xffffffffu, iv, 1);
    float eq = __shfl_up_sync(0xffffffffu, iq, 1);
    if (lane == 0) {
      ev = 0.0;
      eq = 0.0f;
    }
    dsum[lane] = ev;
    fpm[lane] = eq;
  }
  __syncthreads();
  // classify this thread's keys
  double prev = dsum[w] + excl;
  float xmax = fmaxf(fpm[w], pex);  // largest term before the key
  unsigned kk[AX_SM_KPT];
  bool uns[AX_SM_KPT];
  int nu = 0;
  unsigned kl = 0;
#pragma unroll
  for (int i = 0; i < AX_SM_KPT; ++i) {
    const int j = j0 + i;
    const double cur = dsum[w] + excl + c[i];
    const double mg = double(j + 2) * 0x1p-23;
    const double lo = fmax(prev * (1.0 - mg), double(xmax)), hi = cur * (1.0 + mg);
    const int e = binade_index(lo);
    bool safe = j > 0 && binade_index(hi) == e;
    unsigned k = 0;
    if (safe) {
      const double r = double(x[i]) * __longlong_as_double((long long)(23 - e + 1023) << 52);  // x / u, exact
      const double fl = floor(r), fr = r - fl;
      safe = fr != 0.5;
      k = unsigned(fl) + (fr > 0.5 ? 1u : 0u);
    }
    uns[i] = !safe;
    kk[i] = safe ? k : 0u;
    nu += safe ? 0 : 1;
    kl += kk[i];
    eb[j] = (signed char)e;
    prev = cur;
    xmax = fmaxf(xmax, x[i]);
  }
  // positions of the unsafe keys and the k totals before them
  int ni = nu;
  unsigned ki = kl;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int a = __shfl_up_sync(0xffffffffu, ni, off);
    const unsigned b = __shfl_up_sync(0xffffffffu, ki, off);
    if (lane >= off) {
      ni += a;
      ki += b;
    }
  }
  if (lane == 31) {
    nsum[w] = ni;
    ksum[w] = ki;
  }
  __syncthreads();
  if (w == 0) {
    int iv = nsum[lane];
    unsigned ik = ksum[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, iv, off);
      const unsigned b = __shfl_up_sync(0xffffffffu, ik, off);
      if (lane >= off) {
        iv += a;
        ik += b;
      }
    }
    nsum[lane] = iv - nsum[lane];  // exclusive
    ksum[lane] = ik - ksum[lane];
    if (lane == 31) {
      uk[AX_SM_LIST] = ik;  // the total, read as the end of the last run
      s_nuns = iv;
    }
  }
  __syncthreads();
  const int n_uns = s_nuns;
  {
    int idx = nsum[w] + ni - nu;
    unsigned kb = ksum[w] + ki - kl;
#pragma unroll
    for (int i = 0; i < AX_SM_KPT; ++i) {
      if (uns[i]) {
        if (idx < AX_SM_LIST) {
          uq[idx] = j0 + i;
          uk[idx] = kb;
        }
        ++idx;
      }
      kb += kk[i];
    }
  }
  __syncthreads();
  if (n_uns <= AX_SM_LIST) {
    // per unsafe key: its term and the exact value of the safe run after it
    for (int i = t; i < n_uns; i += AX_SM_THREADS) {
      const int q = uq[i];
      const unsigned kend = i + 1 < n_uns ? uk[i + 1] : uk[AX_SM_LIST];
      const unsigned K = kend - uk[i];
      xr[i] = make_float2(ps[q], K != 0u ? ldexpf(float(K), int(eb[min(q + 1, 4095)]) - 23) : 0.0f);
    }
    __syncthreads();
    if (t == 0) {
      float s = 0.0f;
      for (int i = 0; i < n_uns; ++i) {
        const float2 v = xr[i];
        s = __fadd_rn(__fadd_rn(s, v.x), v.y);
      }
      s_sum = s;
    }
  } else if (t == 0) {
    float s = 0.0f;
    for (int j = 0; j < kr.count; ++j) s = __fadd_rn(s, ps[j]);
    s_sum = s;
  }
  __syncthreads();
  const float sum = s_sum;
  float* r = rprob + (size_t(m) * H + h) * cap;
  for (int j = t; j < kr.count; j += AX_SM_THREADS) r[j] = __fdiv_rn(ps[j], sum);
}

// One chain warp's pass over a full stage: out += fround(r_j * v_j) key by
// key.  Keys go in blocks of 16: the block's probabilities as four
// broadcast 16-byte reads and its values one conflict-free word per lane,
// all loaded before the block's adds.
__device__ __forceinline__ float pv_stage_full(const float4* __restrict__ r4, const float* __restrict__ v, float acc) {
#pragma unroll 4
  for (int blk = 0; blk < AX_PV_TC / 16; ++blk) {
    float4 pr[4];
    float vv[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) pr[i] = r4[blk * 4 + i];
#pragma unroll
    for (int i = 0; i < 16; ++i) vv[i] = v[(blk * 16 + i) * AX_PV_DS];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc = __fadd_rn(acc, __fmul_rn(pr[i].x, vv[4 * i]));
      acc = __fadd_rn(acc, __fmul_rn(pr[i].y, vv[4 * i + 1]));
      acc = __fadd_rn(acc, __fmul_rn(pr[i].z, vv[4 * i + 2]));
      acc = __fadd_rn(acc, __fmul_rn(pr[i].w, vv[4 * i + 3]));
    }
  }
  return acc;
}

// One 2-D TMA tile load (this CTA only): box at element (x, y) of `map` into
// this CTA's shared memory, completion on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// vmap: the V cache as a 2-D f32 tensor [cap slots][KVH * 256], box [256][32].
// CW chain warps (one query vector each) share a CTA's V stages; the
// launcher picks the fewest whose grid fits one CTA per SM.
template <int CW>
__global__ void __launch_bounds__(32 * (CW + 1)) hc_attx_pv_kernel(const __grid_constant__ CUtensorMap vmap,
                                                                   const float* __restrict__ rprob,
                                                                   const float* __restrict__ vc,
                                                                   const int32_t* __restrict__ pos, int M, int H,
                                                                   int KVH, int cap, float* __restrict__ out16,
                                                                   int* err) {
  constexpr int AX_PV_QG = CW;  // query vectors per CTA
  constexpr int AX_PV_STAGE = pv_stage_floats(AX_PV_QG);
  extern __shared__ __align__(128) float pv_smem[];  // [NS][AX_PV_STAGE]
  __shared__ __align__(8) uint64_t full[AX_PV_NS], empty[AX_PV_NS];
  constexpr int SLICES = 256 / AX_PV_DS;  // dim slices per KV head
  const int kvh = int(blockIdx.x) / SLICES, ds = int(blockIdx.x) % SLICES, qg = int(blockIdx.y);
  const int lane = int(threadIdx.x) & 31, warp = int(threadIdx.x) >> 5;
  const int G = H / KVH, NQ = M * G;
  const int nq = min(AX_PV_QG, NQ - qg * AX_PV_QG);  // query vectors of this group
  pdl_trigger();
  const KeyRange kr = key_range(pos, M, cap);
  const int nchunk = (kr.count + AX_PV_TC - 1) / AX_PV_TC;
  if (threadIdx.x == 0) {
    for (int s = 0; s < AX_PV_NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CW);
    }
  }
  __syncthreads();
  pdl_wait();  // the probabilities (previous launch) and this step's V rows (two launches back)
  if (warp == CW) {
    // producer: stage c % NS holds keys [256c, 256c + n); it is refilled once
    // the chain warps have released it
    int y0 = kr.start;  // slot of the stage's first key
    int issued = 0;
    bool ok = true;
    for (int c = 0, s = 0, ph = 0; c < nchunk; ++c) {
      if (c >= AX_PV_NS && !mbar_wait_parity_sleep(&empty[s], uint32_t(ph ^ 1), err)) {
        ok = false;
        break;
      }
      const int j0 = c * AX_PV_TC, n = min(AX_PV_TC, kr.count - j0);
      const int n4 = (n + 3) & ~3;  // probability rows are padded to 16 bytes (cap is a multiple of 64)
      float* vs = pv_smem + size_t(s) * AX_PV_STAGE;
      float* ps = vs + AX_PV_TC * AX_PV_DS;
      const bool wraps = y0 + n > cap;
      // the tile load always moves the whole box (rows past cap read as zeros)
      constexpr uint32_t ROWB = AX_PV_DS * 4;
      const uint32_t vbytes = wraps ? uint32_t(n) * ROWB : uint32_t(AX_PV_TC) * ROWB;
      if (lane == 0) {
        mbar_expect_tx(&full[s], vbytes + uint32_t(nq * n4) * 4u);
        if (!wraps) tma_load_2d(vs, &vmap, kvh * 256 + ds * AX_PV_DS, y0, &full[s]);
      }
      __syncwarp();
      if (wraps) {
        for (int jj = lane; jj < n; jj += 32) {
          const int sl = y0 + jj < cap ? y0 + jj : y0 + jj - cap;
          bulk_copy_g2s(vs + jj * AX_PV_DS, vc + (size_t(sl) * KVH + kvh) * 256 + ds * AX_PV_DS, ROWB, &full[s]);
        }
      }
      y0 += AX_PV_TC;
      if (y0 >= cap) y0 -= cap;
      if (lane < nq) {
        const int qw = qg * AX_PV_QG + lane, mm = qw / G, hh = kvh * G + qw % G;
        bulk_copy_g2s(ps + lane * AX_PV_TC, rprob + (size_t(mm) * H + hh) * cap + j0, uint32_t(n4) * 4u, &full[s]);
      }
      ++issued;
      if (++s == AX_PV_NS) {
        s = 0;
        ph ^= 1;
      }
    }
    if (!ok)  // let the copies in flight land before the CTA exits
      for (int c = max(0, issued - AX_PV_NS); c < issued; ++c)
        mbar_wait_parity(&full[c % AX_PV_NS], uint32_t(c / AX_PV_NS) & 1u, nullptr);
    return;
  }
  // chain warps: query vector qg * QG + warp, lane = dim ds * 32 + lane
  const bool active = warp < nq;
  float acc = 0.0f;
  bool ok = true;
  for (int c = 0, s = 0, ph = 0; c < nchunk; ++c) {
    if (ok && !mbar_wait_parity_sleep(&full[s], uint32_t(ph), err)) ok = false;
    if (ok && active) {
      const float* vs = pv_smem + size_t(s) * AX_PV_STAGE;
      const float* r = vs + AX_PV_TC * AX_PV_DS + warp * AX_PV_TC;
      const int n = min(AX_PV_TC, kr.count - c * AX_PV_TC);
      if (n == AX_PV_TC) {
        acc = pv_stage_full(reinterpret_cast<const float4*>(r), vs + lane, acc);
      } else {
        for (int jj = 0; jj < n; ++jj) acc = __fadd_rn(acc, __fmul_rn(r[jj], vs[jj * AX_PV_DS + lane]));
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (++s == AX_PV_NS) {
      s = 0;
      ph ^= 1;
    }
  }
  if (active) {
    const int qi = qg * AX_PV_QG + warp, m = qi / G, h = kvh * G + qi % G;
    out16[(size_t(m) * H + h) * 256 + ds * AX_PV_DS + lane] = round_f16_ts(acc);
  }
}

}  // namespace

size_t attx_scores_smem_bytes(int M, int H, int KVH) {
  return sizeof(float) * (size_t(AX_CH) * AX_KSTRIDE + size_t(M) * (H / KVH) * 256);
}

// scores [M][H][cap], then the probabilities [M][H][cap]
size_t attx_scratch_floats(int M, int H, int cap) { return 2 * size_t(M) * H * cap; }

template <typename... KArgs, typename... Args>
static cudaError_t pdl_launch_x(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
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

// cuTensorMapEncodeTiled through the runtime's driver entry point (the
// library does not link the driver library itself).
static cudaError_t encode_v_map(CUtensorMap* map, const float* vc, int KVH, int cap) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static cudaError_t got = cudaSuccess;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q{};
    got = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&encode), cudaEnableDefault, &q);
    if (got == cudaSuccess && (q != cudaDriverEntryPointSuccess || !encode)) got = cudaErrorSymbolNotFound;
  });
  if (got != cudaSuccess) return got;
  const cuuint64_t dims[2] = {cuuint64_t(KVH) * 256, cuuint64_t(cap)};
  const cuuint64_t strides[1] = {cuuint64_t(KVH) * 256 * sizeof(float)};
  const cuuint32_t box[2] = {AX_PV_DS, AX_PV_TC};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(vc), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

static size_t pv_smem_bytes(int qg) { return sizeof(float) * AX_PV_NS * size_t(pv_stage_floats(qg)); }

template <int CW>
static cudaError_t pv_set_smem() {
  return cudaFuncSetAttribute(hc_attx_pv_kernel<CW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(pv_smem_bytes(CW)));
}

template <int CW>
static cudaError_t pv_launch(int slices, int NQ, cudaStream_t st, const CUtensorMap& vmap, const float* rprob,
                             const float* vc, const int32_t* pos, int M, int H, int KVH, int cap, float* out16,
                             int* err) {
  return pdl_launch_x(hc_attx_pv_kernel<CW>, dim3(slices, (NQ + CW - 1) / CW), dim3(32 * (CW + 1)), pv_smem_bytes(CW),
                      st, vmap, rprob, vc, pos, M, H, KVH, cap, out16, err);
}

cudaError_t launch_attention_exact(const float* q, const float* kraw, const float* vraw, const float* qnw,
                                   const float* knw, const double* cos_t, const double* sin_t, double eps, bool own_kv,
                                   float* kc, float* vc, const int32_t* pos, int M, int H, int KVH, int cap,
                                   float scale, float* scratch, float* out16, cudaStream_t st) {
  if (cap % AX_CH != 0 || cap > 4096) return cudaErrorInvalidValue;
  const size_t smem = attx_scores_smem_bytes(M, H, KVH);
  if (smem > ATT_MAX_SMEM) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr{0};
  const cudaError_t ea = once_per_current_device(attr, [] {
    cudaError_t e = cudaFuncSetAttribute(hc_attx_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(ATT_MAX_SMEM));
    if (e == cudaSuccess) e = pv_set_smem<1>();
    if (e == cudaSuccess) e = pv_set_smem<2>();
    if (e == cudaSuccess) e = pv_set_smem<3>();
    if (e == cudaSuccess) e = pv_set_smem<4>();
    return e;
  });
  if (ea != cudaSuccess) return ea;
  const int chunks = cap / AX_CH;
  float* scores = scratch;
  float* rprob = scores + size_t(M) * H * cap;
  cudaError_t e = pdl_launch_x(hc_attx_scores_kernel, dim3(chunks, KVH), dim3(256), smem, st, q, kraw, vraw, qnw,
                               knw, cos_t, sin_t, eps, int(own_kv), kc, vc, pos, M, H, KVH, cap, scale, scores);
  if (e != cudaSuccess) return e;
  e = pdl_launch_x(hc_attx_softmax_kernel, dim3(M * H), dim3(AX_SM_THREADS), 0, st, scores, pos, M, H, cap, rprob);
  if (e != cudaSuccess) return e;
  const int NQ = M * (H / KVH);
  CUtensorMap vmap;
  e = encode_v_map(&vmap, vc, KVH, cap);
  if (e != cudaSuccess) return e;
  // the fewest chain warps (query vectors) per CTA whose grid fits one CTA per SM
  const int slices = KVH * (256 / AX_PV_DS);
  int cw = 1;
  while (cw < AX_PV_CW_MAX && slices * ((NQ + cw - 1) / cw) > sm_count()) ++cw;
  int* err = device_status_word();
  switch (cw) {
    case 1: return pv_launch<1>(slices, NQ, st, vmap, rprob, vc, pos, M, H, KVH, cap, out16, err);
    case 2: return pv_launch<2>(slices, NQ, st, vmap, rprob, vc, pos, M, H, KVH, cap, out16, err);
    case 3: return pv_launch<3>(slices, NQ, st, vmap, rprob, vc, pos, M, H, KVH, cap, out16, err);
    default: return pv_launch<4>(slices, NQ, st, vmap, rprob, vc, pos, M, H, KVH, cap, out16, err);
  }
}

}  // namespace hc

