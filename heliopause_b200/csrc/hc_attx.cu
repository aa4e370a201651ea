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
//                          4096-term sequential sum (one warp, exact
//                          prefix scans between its binade changes), the
//                          divisions;
//   hc_attx_pv_kernel      grid (KV head x 32-dim slice, groups of 4 query
//                          vectors): one sequential chain per (query, dim)
//                          over all keys, then the TS f16 cast of the output
//                          (castF16Rows, layers.ts:982-988).
// The Q8_K quantization of the cast output for the O projection follows as
// its own launch.
#include <cmath>

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
constexpr int AX_PV_QG = 4;          // query vectors per PV CTA (one warp each)
constexpr int AX_PV_TC = 256;        // keys per staged V chunk
constexpr int AX_PV_NS = 4;          // V chunks in flight (a 4-stage ring: 96 KB of copies ahead of the chain)

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
  bool any = false, fresh = false;
  for (int t = 0; t < AX_CH; ++t) {
    const int j = (t0 + t - kr.start + cap) % cap;
    any |= j < kr.count;
  }
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
  constexpr int U = 4;  // chains per pass
  for (int q0 = ql; q0 < NQ; q0 += AX_QL * U) {
    float dot[U];
#pragma unroll
    for (int u = 0; u < U; ++u) dot[u] = 0.0f;
#pragma unroll 2
    for (int i4 = 0; i4 < HD / 4; ++i4) {
      const float4 b = kv[i4];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int qi = q0 + AX_QL * u;
        if (qi < NQ) {
          const float4 a = reinterpret_cast<const float4*>(qs + qi * HD)[i4];
          dot[u] = __fadd_rn(dot[u], __fmul_rn(a.x, b.x));
          dot[u] = __fadd_rn(dot[u], __fmul_rn(a.y, b.y));
          dot[u] = __fadd_rn(dot[u], __fmul_rn(a.z, b.z));
          dot[u] = __fadd_rn(dot[u], __fmul_rn(a.w, b.w));
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int qi = q0 + AX_QL * u;
      if (qi < NQ && key) {
        const int m = qi / G, h = kvh * G + qi % G;
        // mask 0 where the key is visible: fround(fround(dot * scale) + 0)
        scores[(size_t(m) * H + h) * cap + j] =
            kpos <= pos[m] ? __fadd_rn(__fmul_rn(dot[u], scale), 0.0f) : -INFINITY;
      }
    }
  }
}

// The sequential f32 sum  s = fround(s + v[j]), j = 0 .. n-1, s from +0, of
// non-negative finite terms, bit for bit, by one warp (every lane returns it).
// While the running sum stays in one binade its grid is fixed (ulp 2^e, the
// subnormal grid 2^-149 included), s = M * 2^e with integer M < 2^24, and a
// step adds the term rounded to that grid, k = RN(v / 2^e) -- a plain integer
// -- so a run of steps is an integer prefix sum.  The warp takes 8 terms per
// lane (256 in sequence order), scans the k's and commits every step up to the
// first one whose rounding the grid does not decide: an exact tie (its
// direction depends on the parity of the running sum) or a sum reaching the
// next binade.  That step is done with one f32 add on the committed sum, and
// the scan resumes after it.
__device__ float seq_sum_nonneg_warp(const float* __restrict__ v, int n, int lane) {
  constexpr int PER = 8;
  float s = 0.0f;
  int j = 0;
  while (j < n) {
    const uint32_t ex = (__float_as_uint(s) >> 23) & 0xffu;
    const int e = ex <= 1u ? -149 : int(ex) - 150;  // ulp of s (and of [0, 2^-125))
    const double M = ldexp(double(s), -e);          // the integer significand on that grid
    const double scale = ldexp(1.0, -e);
    const int base = j + PER * lane;
    uint32_t k[PER];
    double q[PER];
    bool bad[PER];
    uint32_t local = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int idx = base + i;
      q[i] = idx < n ? double(v[idx]) * scale : 0.0;  // exact: a power-of-two scaling
      const double fl = floor(q[i]);
      bad[i] = q[i] >= 16777216.0 || q[i] - fl == 0.5;
      k[i] = bad[i] ? 0u : uint32_t(floor(q[i] + 0.5));
      local += k[i];
    }
    uint32_t incl = local;  // steps before the first non-committable one stay below 2^24
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += t;
    }
    uint32_t run = incl - local;
    int first = PER;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      if (first == PER && base + i < n) {
        // the exact pre-rounding value on the grid: M + run + q
        if (bad[i] || (M + double(run)) + q[i] >= 16777215.5) first = i;
        else run += k[i];
      }
    }
    const unsigned m = __ballot_sync(0xffffffffu, first < PER);
    if (m == 0u) {
      const uint32_t tot = __shfl_sync(0xffffffffu, incl, 31);
      s = float(ldexp(M + double(tot), e));
      j += 32 * PER;
    } else {
      const int fl_lane = __ffs(m) - 1;
      const int fi = __shfl_sync(0xffffffffu, first, fl_lane);
      const uint32_t committed = __shfl_sync(0xffffffffu, run, fl_lane);
      const int idx = j + PER * fl_lane + fi;
      s = __fadd_rn(float(ldexp(M + double(committed), e)), v[idx]);
      j = idx + 1;
    }
  }
  return s;
}

__global__ void __launch_bounds__(AX_SM_THREADS) hc_attx_softmax_kernel(const float* __restrict__ scores,
                                                                        const int32_t* __restrict__ pos, int M, int H,
                                                                        int cap, float* __restrict__ rprob) {
  __shared__ float ps[4096];
  __shared__ float red[AX_SM_THREADS / 32];
  __shared__ float s_sum;
  const int m = int(blockIdx.x) / H, h = int(blockIdx.x) % H;
  pdl_trigger();
  const KeyRange kr = key_range(pos, M, cap);
  pdl_wait();
  // the max over every key (exact and order-free; -inf never wins over a
  // visible key, and every token sees its own key)
  const float* sc = scores + (size_t(m) * H + h) * cap;
  float mx = -INFINITY;
  for (int j = int(threadIdx.x); j < kr.count; j += int(blockDim.x)) {
    const float s = sc[j];
    ps[j] = s;
    mx = fmaxf(mx, s);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = -INFINITY;
  for (int w = 0; w < int(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
  for (int j = int(threadIdx.x); j < kr.count; j += int(blockDim.x)) {
    const float s = ps[j];
    ps[j] = s == -INFINITY ? 0.0f : float(exp(double(__fsub_rn(s, mx))));
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // the sequential sum (lib.rs:627-635), by one warp
    const float sum = seq_sum_nonneg_warp(ps, kr.count, int(threadIdx.x));
    if (threadIdx.x == 0) s_sum = sum;
  }
  __syncthreads();
  const float sum = s_sum;
  float* r = rprob + (size_t(m) * H + h) * cap;
  for (int j = int(threadIdx.x); j < kr.count; j += int(blockDim.x)) r[j] = __fdiv_rn(ps[j], sum);
}

__global__ void __launch_bounds__(32 * AX_PV_QG) hc_attx_pv_kernel(const float* __restrict__ rprob,
                                                                   const float* __restrict__ vc,
                                                                   const int32_t* __restrict__ pos, int M, int H,
                                                                   int KVH, int cap, float* __restrict__ out16) {
  extern __shared__ __align__(16) float pv_smem[];
  float (*vs)[AX_PV_TC][32] = reinterpret_cast<float (*)[AX_PV_TC][32]>(pv_smem);  // [NS][TC][32]
  float (*rs)[AX_PV_QG][AX_PV_TC] =
      reinterpret_cast<float (*)[AX_PV_QG][AX_PV_TC]>(pv_smem + AX_PV_NS * AX_PV_TC * 32);  // [NS][QG][TC]
  const int kvh = int(blockIdx.x) >> 3, ds = int(blockIdx.x) & 7, qg = int(blockIdx.y);
  const int lane = int(threadIdx.x) & 31, warp = int(threadIdx.x) >> 5;
  const int G = H / KVH, NQ = M * G;
  const int qi = qg * AX_PV_QG + warp;
  pdl_trigger();
  const KeyRange kr = key_range(pos, M, cap);
  const int nchunk = (kr.count + AX_PV_TC - 1) / AX_PV_TC;
  pdl_wait();  // the probabilities (previous launch) and this step's V rows (two launches back)
  auto load_chunk = [&](int c, int buf) {
    const int j0 = c * AX_PV_TC, n = min(AX_PV_TC, kr.count - j0);
    // V: 8 sixteen-byte pieces per key (this slice's 32 dims)
    for (int i = int(threadIdx.x); i < n * 8; i += int(blockDim.x)) {
      const int jj = i >> 3, pc = i & 7;
      const int slot = (kr.start + j0 + jj) % cap;
      cp_async16(&vs[buf][jj][4 * pc], vc + (size_t(slot) * KVH + kvh) * 256 + ds * 32 + 4 * pc);
    }
    // probabilities of the group's query vectors
    for (int i = int(threadIdx.x); i < AX_PV_QG * (AX_PV_TC / 4); i += int(blockDim.x)) {
      const int w = i / (AX_PV_TC / 4), pc = i % (AX_PV_TC / 4);
      const int qw = qg * AX_PV_QG + w;
      if (qw < NQ && 4 * pc < n) {
        const int mm = qw / G, hh = kvh * G + qw % G;
        const float* src = rprob + (size_t(mm) * H + hh) * cap + j0 + 4 * pc;
        if (4 * pc + 4 <= n) {
          cp_async16(&rs[buf][w][4 * pc], src);
        } else {
          for (int e = 0; 4 * pc + e < n; ++e) rs[buf][w][4 * pc + e] = src[e];
        }
      }
    }
    cp_async_commit();
  };
  float acc = 0.0f;
  // a ring of NS chunks: chunks c + 1 .. c + NS - 1 are in flight while the
  // chain walks chunk c (one commit group per chunk, empty past the end)
  for (int c = 0; c < AX_PV_NS - 1; ++c) {
    if (c < nchunk) load_chunk(c, c);
    else cp_async_commit();
  }
  for (int c = 0; c < nchunk; ++c) {
    const int buf = c % AX_PV_NS;
    if (c + AX_PV_NS - 1 < nchunk) load_chunk(c + AX_PV_NS - 1, (c + AX_PV_NS - 1) % AX_PV_NS);
    else cp_async_commit();
    asm volatile("cp.async.wait_group %0;" ::"n"(AX_PV_NS - 1) : "memory");
    __syncthreads();
    const int n = min(AX_PV_TC, kr.count - c * AX_PV_TC);
    if (qi < NQ) {
      const float* r = rs[buf][warp];
      int jj = 0;
      for (; jj + 4 <= n; jj += 4) {
        const float4 p4 = *reinterpret_cast<const float4*>(r + jj);
        acc = __fadd_rn(acc, __fmul_rn(p4.x, vs[buf][jj][lane]));
        acc = __fadd_rn(acc, __fmul_rn(p4.y, vs[buf][jj + 1][lane]));
        acc = __fadd_rn(acc, __fmul_rn(p4.z, vs[buf][jj + 2][lane]));
        acc = __fadd_rn(acc, __fmul_rn(p4.w, vs[buf][jj + 3][lane]));
      }
      for (; jj < n; ++jj) acc = __fadd_rn(acc, __fmul_rn(r[jj], vs[buf][jj][lane]));
    }
    __syncthreads();  // the buffer is refilled NS - 1 chunks later
  }
  if (qi < NQ) {
    const int m = qi / G, h = kvh * G + qi % G;
    out16[(size_t(m) * H + h) * 256 + ds * 32 + lane] = round_f16_ts(acc);
  }
}

}  // namespace

__global__ void hc_seq_sum_test_kernel(const float* v, int n, float* out) {
  const float s = seq_sum_nonneg_warp(v, n, int(threadIdx.x));
  if (threadIdx.x == 0) *out = s;
}

size_t attx_scores_smem_bytes(int M, int H, int KVH) {
  return sizeof(float) * (size_t(AX_CH) * AX_KSTRIDE + size_t(M) * (H / KVH) * 256);
}

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

cudaError_t launch_attention_exact(const float* q, const float* kraw, const float* vraw, const float* qnw,
                                   const float* knw, const double* cos_t, const double* sin_t, double eps, bool own_kv,
                                   float* kc, float* vc, const int32_t* pos, int M, int H, int KVH, int cap,
                                   float scale, float* scratch, float* out16, cudaStream_t st) {
  if (cap % AX_CH != 0 || cap > 4096) return cudaErrorInvalidValue;
  const size_t smem = attx_scores_smem_bytes(M, H, KVH);
  if (smem > ATT_MAX_SMEM) return cudaErrorInvalidValue;
  constexpr size_t pv_smem = sizeof(float) * AX_PV_NS * AX_PV_TC * (32 + AX_PV_QG);
  static std::atomic<uint64_t> attr{0};
  const cudaError_t ea = once_per_current_device(attr, [] {
    cudaError_t e = cudaFuncSetAttribute(hc_attx_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(ATT_MAX_SMEM));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(hc_attx_pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(pv_smem));
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
  return pdl_launch_x(hc_attx_pv_kernel, dim3(KVH * 8, (NQ + AX_PV_QG - 1) / AX_PV_QG), dim3(32 * AX_PV_QG), pv_smem,
                      st, rprob, vc, pos, M, H, KVH, cap, out16);
}

}  // namespace hc

// Test hook (not part of the public header): runs the softmax's warp-scan
// sequential sum over n non-negative device floats into *d_out, so tests can
// compare it with a plain sequential f32 sum on chosen inputs.
extern "C" int hc_test_seq_sum(const float* d_v, int n, float* d_out) {
  hc::hc_seq_sum_test_kernel<<<1, 32>>>(d_v, n, d_out);
  return cudaDeviceSynchronize() == cudaSuccess ? 0 : 4;
}
