// hc_persist.cu -- the decode step (M = 1) of all decoder layers as ONE
// persistent cooperative kernel.
//
// Replaces, for a single token, the per-layer kernel chain of hc_model.cu
// (norm+quant -> QKV GEMV -> QK-norm/RoPE/KV write -> split-KV attention ->
// combine -> O GEMV -> residual+norm+quant -> gate/up GEMV -> GEGLU+quant ->
// down GEMV), i.e. forwardAttentionLayer + forwardFfn of the WASM provider
// (packages/engine/src/runner/wasm/layers.ts:161-473), with the same
// arithmetic as the per-kernel path (hc_decode.cu, hc_gemv_body.cuh).
//
// Why: at M = 1 a layer streams ~79 MB of weights but its ten dependent
// kernels each pay launch, ramp and drain latency; the per-kernel step reaches
// ~21% of HBM bandwidth.  Here one CTA per SM lives for the whole step:
//
//   * Weight stream.  Every warp owns a ring of P_SLOTS shared-memory slots and
//     walks a fixed sequence of "units" (one 256-block of one 32-row weight
//     tile, or 4 KV tokens of one KV head) across all stages and layers.  Lane
//     0 refills a slot with a bulk copy (cp.async.bulk, mbarrier completion)
//     as soon as the warp has consumed it, so the copies run up to P_SLOTS
//     units ahead of the computation -- across stage boundaries, i.e. while
//     the CTA waits for the previous stage's results.
//   * Work split.  A GEMV stage's units are numbered tile-major; CTA c takes
//     the contiguous range [U*c/G, U*(c+1)/G) and its warps split that range
//     contiguously.  Each CTA reduces its warps' per-tile row sums in warp
//     order and stores one partial per (tile, CTA); the consumer sums a tile's
//     partials in CTA order.  Every result is deterministic.
//   * Dependencies.  Each (layer, stage) has a global counter; a CTA adds 1
//     after its stage outputs are stored (fence, then atomic add) and the next
//     stage's CTAs wait until the counter reaches its producer count (thread 0
//     polls with ld.acquire.gpu, bounded by %globaltimer; a timeout sets the
//     status word and an abort word, every CTA then drains its copies and
//     exits).  The launch is cooperative, so all CTAs are co-resident.
//   * Prologues instead of kernels.  The RMSNorms + residual adds and the
//     Q8_K quantization of a GEMV's input are recomputed by every CTA from L2
//     (a few tens of KB) instead of being separate launches; the QK-norm and
//     RoPE of the queries are recomputed by every attention CTA.
//
// Stage sequence per layer (producer count of its counter in brackets):
//   QKV   [grid]  prologue: x_l = H1 + rmsnorm(down_{l-1}) (CTA 0 stores X),
//                 q8(rmsnorm(x_l) * w_attn); units of Q|K|V
//   ATT   [grid]  queries (QK-norm, RoPE, Rust f16 rounding); the CTA whose
//                 tokens hold `pos` computes the new K/V row (own-KV layers)
//                 or reads it (shared-KV layers) and overrides the staged
//                 row; online softmax over 4-token units; per-CTA partial
//   COMB  [H]     CTA h merges head h's partials, TS f16 cast, Q8_K block h
//   O     [grid]  units of O on the staged attention records
//   GU    [grid]  prologue: h1 = x_l + rmsnorm(o) (CTA 0 stores H1),
//                 q8(rmsnorm(h1) * w_ffn); units of gate|up
//   ACT   [F/2048] CTA c, warp w: GEGLU of 256-block 8c+w, Q8_K
//   DOWN  [grid]  units of down on the staged activation records
// and at the end CTA 0 stores the final residual x_L in X.
#include <cooperative_groups.h>

#include "hc_bulk.cuh"
#include "hc_common.cuh"
#include "hc_decmath.cuh"
#include "hc_gemv_body.cuh"
#include "hc_kernels.cuh"
#include "hc_persist.cuh"
#include "hc_q8.cuh"

namespace hc {

namespace {

// ---- shared memory map (bytes) ----------------------------------------------------
constexpr int SM_RING = 0;
constexpr int SM_ACT = SM_RING + P_WARPS * P_SLOTS * P_SLOT_BYTES;
constexpr int SM_RED = SM_ACT + P_ACT_BYTES;                       // [P_WARPS][P_WARP_TILES][32] f32
constexpr int SM_BARS = SM_RED + P_WARPS * P_WARP_TILES * 32 * 4;  // [P_WARPS][P_SLOTS] mbarriers
constexpr int SM_STAGE = SM_BARS + P_WARPS * P_SLOTS * 8;          // [P_WARPS][256] q8 staging
constexpr int SM_QS = SM_STAGE + P_WARPS * 256;                    // [P_MAX_G][256] f32 queries
constexpr int SM_FRESH = SM_QS + P_MAX_G * 256 * 4;                // new K row, new V row [2][256] f32
constexpr int SM_MISC = SM_FRESH + 2 * 256 * 4;                    // reduction scratch + small ints
constexpr int SM_TOTAL = SM_MISC + 64 * 8;
static_assert(SM_TOTAL <= 232448, "exceeds the 227 KB per-CTA shared memory");
static_assert(P_ATT_WARPS * P_ATT_REC * 4 <= P_ACT_BYTES, "attention merge staging reuses the activation area");

constexpr int RING_STAGES = 5;  // QKV, ATT, O, GU, DOWN: the stages that stream units
constexpr int ST_QKV = 0, ST_ATT = 1, ST_O = 2, ST_GU = 3;

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Thread 0 waits for *ctr >= target; returns false (every thread) if the step
// was aborted or the wait timed out.  Up to ~150 CTAs poll one counter, so the
// poll is a relaxed load with exponential backoff (64..512 ns) and the abort
// word is read every 16 polls; the acquire fence follows the successful poll.
__device__ __forceinline__ bool cta_wait(const PParams& p, const unsigned* ctr, unsigned target) {
  int ok = 1;
  if (threadIdx.x == 0) {
    const unsigned long long t0 = gtimer();
    unsigned ns = 64;
    for (unsigned it = 0; ld_relaxed(ctr) < target; ++it) {
      if ((it & 15) == 15) {
        if (ld_volatile(p.abort_word) != 0) {
          ok = 0;
          break;
        }
        if (gtimer() - t0 > WAIT_LIMIT_NS) {
          atomicExch(p.err, DEVICE_ERR_TIMEOUT);
          atomicExch(p.abort_word, 1);
          ok = 0;
          break;
        }
      }
      __nanosleep(ns);
      if (ns < 512) ns *= 2;
    }
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
  }
  return __syncthreads_and(ok) != 0;
}

// All threads: publish this CTA's stage outputs.
__device__ __forceinline__ void cta_signal(unsigned* ctr) {
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __threadfence();
    atomicAdd(ctr, 1u);
  }
}

__device__ __forceinline__ unsigned* counter(const PParams& p, int layer, int stage) {
  return p.counters + (layer * PS_COUNT + stage) * P_CTR_STRIDE;
}

__device__ __forceinline__ const PGemv& gemv_of(const PLayer& L, int st) {
  return st == ST_QKV ? L.qkv : (st == ST_O ? L.o : (st == ST_GU ? L.gu : L.down));
}


// Read-only plan fields through the non-coherent cache (the plan is never
// written while the kernel runs).
__device__ __forceinline__ int pl_i(const int& v) { return __ldg(&v); }
template <class T>
__device__ __forceinline__ T* pl_p(T* const& v) {
  return reinterpret_cast<T*>(__ldg(reinterpret_cast<const unsigned long long*>(&v)));
}

// Number of per-CTA partials of tile t of a GEMV stage.
__device__ __forceinline__ int gemv_nseg(int B, int U, int t, int grid) {
  return p_cta_of(t * B + B - 1, U, grid) - p_cta_of(t * B, U, grid) + 1;
}

// Sums of a GEMV stage's partials for output rows of the concatenated tile
// list, in CTA order.
// The same for NR rows (rows[i] < 0: skipped, out 0).  Loads are
// unconditional (segment index clamped to the tile's last partial, the extra
// terms added as zero), so the compiler keeps them all in flight; the sums
// run in segment order.
template <int NR>
__device__ __forceinline__ void gemv_rows(const PGemv& g, const int (&rows)[NR], int grid, float (&out)[NR]) {
  const int B = pl_i(g.B), U = pl_i(g.tiles) * B, ms = pl_i(g.maxseg);
  const float* part = pl_p(g.part);
  int n[NR];
  const float* src[NR];
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    const int row = rows[r] >= 0 ? rows[r] : 0, t = row >> 5;
    n[r] = rows[r] >= 0 ? gemv_nseg(B, U, t, grid) : 0;
    src[r] = part + (size_t(t) * ms) * 32 + (row & 31);
    out[r] = 0.0f;
  }
  for (int k0 = 0; k0 < ms; k0 += 4) {
    float v[NR][4];
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int k = 0; k < 4; ++k) v[r][k] = __ldcg(src[r] + min(k0 + k, max(n[r], 1) - 1) * 32);
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int k = 0; k < 4; ++k) out[r] += k0 + k < n[r] ? v[r][k] : 0.0f;
  }
}

// The same for 8 consecutive rows row0..row0+7 (row0 % 8 == 0, one tile),
// float4 loads, unconditional (clamped) as above.
__device__ __forceinline__ void gemv_rows8(const PGemv& g, int row0, int grid, float (&out)[8]) {
  const int B = pl_i(g.B), t = row0 >> 5, n = gemv_nseg(B, pl_i(g.tiles) * B, t, grid), ms = pl_i(g.maxseg);
  const float4* src = reinterpret_cast<const float4*>(pl_p(g.part) + (size_t(t) * ms) * 32 + (row0 & 31));
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = 0.0f;
  for (int k0 = 0; k0 < n; k0 += 4) {
    float4 v[4][2];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int kk = min(k0 + k, n - 1);
      v[k][0] = __ldcg(src + kk * 8);
      v[k][1] = __ldcg(src + kk * 8 + 1);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float z = k0 + k < n ? 1.0f : 0.0f;
      if (k0 + k < n) {
        out[0] += v[k][0].x; out[1] += v[k][0].y; out[2] += v[k][0].z; out[3] += v[k][0].w;
        out[4] += v[k][1].x; out[5] += v[k][1].y; out[6] += v[k][1].z; out[7] += v[k][1].w;
      }
      (void)z;
    }
  }
}

// ---- the per-warp unit stream -------------------------------------------------------

struct StreamCtx {
  const PParams* p;
  int grid, cta, warp, lane;
  int count;     // attention tokens [0, count)
  int att_cpk;   // CTAs per KV head in the attention stage
};

// Unit range [lo, hi) of this warp in ring stage `st` of `layer`.
__device__ __forceinline__ void warp_range(const StreamCtx& x, int layer, int st, int* lo, int* hi) {
  if (st == ST_ATT) {
    const int kvh = x.cta / x.att_cpk, j = x.cta % x.att_cpk;
    *lo = *hi = 0;
    if (kvh >= x.p->KVH || x.warp >= P_ATT_WARPS) return;
    const int nu = (x.count + P_ATT_TOK - 1) / P_ATT_TOK;
    const int c0 = p_range_lo(nu, j, x.att_cpk), c1 = p_range_lo(nu, j + 1, x.att_cpk);
    const int n = c1 - c0;
    *lo = c0 + n * x.warp / P_ATT_WARPS;
    *hi = c0 + n * (x.warp + 1) / P_ATT_WARPS;
    return;
  }
  const PGemv& g = gemv_of(x.p->layers[layer], st);
  const int U = pl_i(g.tiles) * pl_i(g.B);
  const int c0 = p_range_lo(U, x.cta, x.grid), c1 = p_range_lo(U, x.cta + 1, x.grid);
  const int n = c1 - c0;
  *lo = c0 + n * x.warp / P_WARPS;
  *hi = c0 + n * (x.warp + 1) / P_WARPS;
}

// A position in a warp's unit sequence.  For a GEMV stage it carries the
// current weight segment (source address of unit u, unit bytes, end of the
// segment), so that consecutive units -- contiguous in HBM within a segment
// -- need no plan reads; the plan is read at stage and segment boundaries.
struct Cursor {
  int layer, st, u, hi;
  bool done;
  const uint8_t* src;  // GEMV: unit u;  attention: K cache of the layer
  const uint8_t* src2; // attention: V cache of the layer
  int ub;              // GEMV unit bytes
  int seg_hi;          // GEMV: first unit after the current segment
};

__device__ __forceinline__ void cursor_locate(const StreamCtx& x, Cursor& c) {
  const PLayer& L = x.p->layers[c.layer];
  if (c.st == ST_ATT) {
    c.src = reinterpret_cast<const uint8_t*>(pl_p(L.kc));
    c.src2 = reinterpret_cast<const uint8_t*>(pl_p(L.vc));
    return;
  }
  const PGemv& g = gemv_of(L, c.st);
  const int B = pl_i(g.B), tile = c.u / B;
  const int e0 = pl_i(g.tile_end[0]), e1 = pl_i(g.tile_end[1]);
  const int s = tile < e0 ? 0 : (tile < e1 ? 1 : 2);
  const int begin = s == 0 ? 0 : (s == 1 ? e0 : e1);
  const int end = s == 0 ? e0 : (s == 1 ? e1 : pl_i(g.tile_end[2]));
  c.ub = unit_bytes(pl_i(g.type[s]));
  c.seg_hi = end * B;
  c.src = pl_p(g.w[s]) + size_t(c.u - begin * B) * c.ub;
}

__device__ __forceinline__ void cursor_settle(const StreamCtx& x, Cursor& c) {
  bool moved = false;
  while (!c.done && c.u >= c.hi) {
    moved = true;
    if (++c.st == RING_STAGES) {
      c.st = 0;
      if (++c.layer == x.p->nlayers) {
        c.done = true;
        break;
      }
    }
    warp_range(x, c.layer, c.st, &c.u, &c.hi);
  }
  if (moved && !c.done) cursor_locate(x, c);
}

__device__ __forceinline__ Cursor cursor_begin(const StreamCtx& x) {
  Cursor c{0, 0, 0, 0, false, nullptr, nullptr, 0, 0};
  warp_range(x, 0, 0, &c.u, &c.hi);
  if (c.u < c.hi) cursor_locate(x, c);
  cursor_settle(x, c);
  return c;
}

__device__ __forceinline__ void cursor_next(const StreamCtx& x, Cursor& c) {
  ++c.u;
  if (c.u < c.hi) {
    if (c.st == ST_ATT) return;
    if (c.u < c.seg_hi) {
      c.src += c.ub;
      return;
    }
    cursor_locate(x, c);  // next weight of the stage
    return;
  }
  cursor_settle(x, c);
}

// Lane 0: bulk copies of the unit at `c` into `slot`, completing on `bar`.
__device__ __forceinline__ void issue_unit(const StreamCtx& x, const Cursor& c, uint8_t* slot, uint64_t* bar) {
  if (c.st == ST_ATT) {
    const int kvh = x.cta / x.att_cpk, KVH = x.p->KVH;
    const int t0 = c.u * P_ATT_TOK;
    mbar_expect_tx(bar, uint32_t(2 * P_ATT_TOK * 1024));
#pragma unroll
    for (int i = 0; i < P_ATT_TOK; ++i) {
      const size_t off = (size_t(t0 + i) * KVH + kvh) * 1024;
      bulk_copy_g2s(slot + i * 1024, c.src + off, 1024, bar);
      bulk_copy_g2s(slot + (P_ATT_TOK + i) * 1024, c.src2 + off, 1024, bar);
    }
    return;
  }
  mbar_expect_tx(bar, uint32_t(c.ub));
  bulk_copy_g2s(slot, c.src, uint32_t(c.ub), bar);
}

struct Ring {
  uint8_t* base;   // this warp's slots
  uint64_t* bars;  // this warp's barriers
  Cursor issue;    // next unit to issue
  unsigned seq;    // units consumed so far
  unsigned issued; // units issued so far
};

__device__ __forceinline__ uint8_t* ring_slot(const Ring& r, unsigned i) {
  return r.base + (i % P_SLOTS) * P_SLOT_BYTES;
}

// Lane 0 keeps P_SLOTS units in flight.
__device__ __forceinline__ void ring_fill(const StreamCtx& x, Ring& r) {
  while (!r.issue.done && r.issued < r.seq + P_SLOTS) {
    if (x.lane == 0) issue_unit(x, r.issue, ring_slot(r, r.issued), r.bars + (r.issued % P_SLOTS));
    ++r.issued;
    cursor_next(x, r.issue);
  }
}

// Waits for the next unit (the caller knows it was issued).  false on timeout.
__device__ __forceinline__ bool ring_wait(const PParams& p, Ring& r) {
  return mbar_wait_parity(r.bars + (r.seq % P_SLOTS), (r.seq / P_SLOTS) & 1u, p.err);
}

// After the warp has consumed the slot's values (every register loaded from
// it has been used, so its shared-memory reads are complete): release it and
// issue the next unit into it.
__device__ __forceinline__ void ring_release(const StreamCtx& x, Ring& r) {
  __syncwarp();
  ++r.seq;
  ring_fill(x, r);
}

// On abort: wait (bounded) for this warp's copies in flight.
__device__ __forceinline__ void ring_drain(const PParams& p, Ring& r) {
  while (r.seq < r.issued) {
    mbar_wait_parity(r.bars + (r.seq % P_SLOTS), (r.seq / P_SLOTS) & 1u, nullptr);
    ++r.seq;
  }
}

// ---- prologues -------------------------------------------------------------------------

// Quantizes n[] (this thread's 8 values of 256-block `warp + 8*i`) into the
// activation area: plane A records at act, plane B after nb of them.
__device__ __forceinline__ void quant_into(uint8_t* act, uint8_t* stage, const float (&n)[8], int blk, int nb,
                                           int lane) {
  q8k_block_warp(n, lane, stage, act + size_t(blk) * Q8A_REC, act + size_t(nb) * Q8A_REC + size_t(blk) * Q8B_REC);
}

// out[i] = rmsnorm(v) * w over D values held 8 per thread in v[j][8] (block
// warp + 8 j), f64 sums (rmsNormVector, layers.ts:871-885).
template <int NBW>
__device__ __forceinline__ double block_rms_scale(const float (&v)[NBW][8], int nbw, int D, double eps,
                                                  double* scratch) {
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < NBW; ++j)
    if (j < nbw) {
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += double(v[j][i]) * double(v[j][i]);
    }
  ss = block_sum_d(ss, scratch, P_WARPS);
  return 1.0 / sqrt(ss / double(D) + eps);
}


// QKV prologue of layer l: x_l (into X by CTA 0) and q8(rmsnorm(x_l) * w_attn).
// NBW = 256-blocks of the hidden vector per warp (D / 2048).
template <int NBW>
__device__ __forceinline__ void prologue_attn_input(const PParams& p, int l, uint8_t* smem, int grid) {
  constexpr int NBW_MAX = NBW;
  const int D = p.D, nb = D / 256, nbw = NBW;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double* scratch = reinterpret_cast<double*>(smem + SM_MISC);
  float x[NBW_MAX][8];
  const PLayer& L = p.layers[l];
  if (l == 0) {
#pragma unroll
    for (int j = 0; j < NBW_MAX; ++j)
      if (j < nbw) {
        const int e0 = (warp + P_WARPS * j) * 256 + 8 * lane;
#pragma unroll
        for (int i = 0; i < 8; ++i) x[j][i] = __ldcg(p.X + e0 + i);
      }
  } else {
    const PLayer& Lp = p.layers[l - 1];
    float y[NBW_MAX][8];
#pragma unroll
    for (int j = 0; j < NBW_MAX; ++j)
      if (j < nbw) {
        const int e0 = (warp + P_WARPS * j) * 256 + 8 * lane;
        gemv_rows8(Lp.down, e0, grid, y[j]);
      }
    const double sc = block_rms_scale<NBW_MAX>(y, nbw, D, p.eps, scratch);
#pragma unroll
    for (int j = 0; j < NBW_MAX; ++j)
      if (j < nbw) {
        const int e0 = (warp + P_WARPS * j) * 256 + 8 * lane;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float pn = float((double(y[j][i]) * sc) * double(__ldg(Lp.n_post_ffw + e0 + i)));
          x[j][i] = __ldcg(p.H1 + e0 + i) + pn;
        }
        if (blockIdx.x == 0) {
#pragma unroll
          for (int i = 0; i < 8; ++i) p.X[e0 + i] = x[j][i];
        }
      }
  }
  const double sc = block_rms_scale<NBW_MAX>(x, nbw, D, p.eps, scratch);
  uint8_t* act = smem + SM_ACT;
  uint8_t* stage = smem + SM_STAGE + warp * 256;
#pragma unroll
  for (int j = 0; j < NBW_MAX; ++j)
    if (j < nbw) {
      const int blk = warp + P_WARPS * j, e0 = blk * 256 + 8 * lane;
      float n[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) n[i] = float((double(x[j][i]) * sc) * double(__ldg(L.n_attn + e0 + i)));
      quant_into(act, stage, n, blk, nb, lane);
    }
}

// GU prologue of layer l: h1 = x_l + rmsnorm(o) (into H1 by CTA 0) and
// q8(rmsnorm(h1) * w_ffn).
template <int NBW>
__device__ __forceinline__ void prologue_ffn_input(const PParams& p, int l, uint8_t* smem, int grid) {
  constexpr int NBW_MAX = NBW;
  const int D = p.D, nb = D / 256, nbw = NBW;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double* scratch = reinterpret_cast<double*>(smem + SM_MISC);
  const PLayer& L = p.layers[l];
  float y[NBW_MAX][8], h[NBW_MAX][8];
#pragma unroll
  for (int j = 0; j < NBW_MAX; ++j)
    if (j < nbw) {
      const int e0 = (warp + P_WARPS * j) * 256 + 8 * lane;
      gemv_rows8(L.o, e0, grid, y[j]);
    }
  const double sc = block_rms_scale<NBW_MAX>(y, nbw, D, p.eps, scratch);
#pragma unroll
  for (int j = 0; j < NBW_MAX; ++j)
    if (j < nbw) {
      const int e0 = (warp + P_WARPS * j) * 256 + 8 * lane;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float pn = float((double(y[j][i]) * sc) * double(__ldg(L.n_post_attn + e0 + i)));
        h[j][i] = __ldcg(p.X + e0 + i) + pn;
      }
      if (blockIdx.x == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) p.H1[e0 + i] = h[j][i];
      }
    }
  const double sc2 = block_rms_scale<NBW_MAX>(h, nbw, D, p.eps, scratch);
  uint8_t* act = smem + SM_ACT;
  uint8_t* stage = smem + SM_STAGE + warp * 256;
#pragma unroll
  for (int j = 0; j < NBW_MAX; ++j)
    if (j < nbw) {
      const int blk = warp + P_WARPS * j, e0 = blk * 256 + 8 * lane;
      float n[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) n[i] = float((double(h[j][i]) * sc2) * double(__ldg(L.n_ffn + e0 + i)));
      quant_into(act, stage, n, blk, nb, lane);
    }
}

// Copies `bytes` of Q8_K records written by other CTAs into the activation area.
__device__ __forceinline__ void stage_records(uint8_t* dst, const uint8_t* src, int bytes) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = __ldcg(s + i);
}

// ---- GEMV stage ------------------------------------------------------------------------

// Streams this warp's units of GEMV stage `st`, reduces the CTA's per-tile row
// sums and stores its partials.  Activation records are at SM_ACT: both planes
// (nb records each, plane B after plane A) or one plane (`single_plane`).
__device__ __forceinline__ bool gemv_stage(const StreamCtx& x, Ring& r, const PGemv& g, uint8_t* smem, bool single_plane) {
  const int warp = x.warp, lane = x.lane, B = pl_i(g.B), U = pl_i(g.tiles) * B;
  const int te0 = pl_i(g.tile_end[0]), te1 = pl_i(g.tile_end[1]);
  const int ty0 = pl_i(g.type[0]), ty1 = pl_i(g.type[1]), ty2 = pl_i(g.type[2]);
  const int maxseg = pl_i(g.maxseg);
  float* const part = pl_p(g.part);
  int lo, hi;
  {
    const int c0 = p_range_lo(U, x.cta, x.grid), c1 = p_range_lo(U, x.cta + 1, x.grid), n = c1 - c0;
    lo = c0 + n * warp / P_WARPS;
    hi = c0 + n * (warp + 1) / P_WARPS;
  }
  uint8_t* act = smem + SM_ACT;
  ActSlice as;
  if (single_plane) {
    as = ActSlice{act, act, B, 0};
  } else {
    as = ActSlice{act, act + size_t(B) * Q8A_REC, B, 0};
  }
  float* red = reinterpret_cast<float*>(smem + SM_RED) + warp * P_WARP_TILES * 32;
  int* wt = reinterpret_cast<int*>(smem + SM_MISC + 32 * 8);  // [P_WARPS][2]: first tile, count
  const int wt0 = lo / B;
  if (lane == 0) {
    wt[2 * warp] = wt0;
    wt[2 * warp + 1] = hi > lo ? (hi - 1) / B - wt0 + 1 : 0;
  }
  bool ok = true;
  float acc[1] = {0.0f};
  int cur = wt0;
  // Two units per iteration when they belong to the same tile: two
  // independent dot chains in flight; the sums are added in unit order, as
  // one at a time.
#pragma unroll 1
  for (int u = lo; u < hi;) {
    const int tile = u / B, blk = u - tile * B;
    if (tile != cur) {
      red[(cur - wt0) * 32 + lane] = acc[0];
      acc[0] = 0.0f;
      cur = tile;
    }
    const int type = tile < te0 ? ty0 : (tile < te1 ? ty1 : ty2);
    const bool pair = u + 1 < hi && blk + 1 < B;
    if (!ring_wait(*x.p, r)) {
      ok = false;
      break;
    }
    const uint8_t* unit0 = ring_slot(r, r.seq);
    if (pair) {
      if (!mbar_wait_parity(r.bars + ((r.seq + 1) % P_SLOTS), ((r.seq + 1) / P_SLOTS) & 1u, x.p->err)) {
        ok = false;
        break;
      }
      const uint8_t* unit1 = ring_slot(r, r.seq + 1);
      float d0, d1;
      if (type == TYPE_Q4_K) {
        d0 = q4k_smem_dot(unit0, blk, as, lane);
        d1 = q4k_smem_dot(unit1, blk + 1, as, lane);
      } else {
        d0 = q6k_smem_dot(unit0, blk, as, lane);
        d1 = q6k_smem_dot(unit1, blk + 1, as, lane);
      }
      acc[0] += d0;
      acc[0] += d1;
      ring_release(x, r);
      ring_release(x, r);
      u += 2;
    } else {
      acc[0] += type == TYPE_Q4_K ? q4k_smem_dot(unit0, blk, as, lane) : q6k_smem_dot(unit0, blk, as, lane);
      ring_release(x, r);
      u += 1;
    }
  }
  if (hi > lo) red[(cur - wt0) * 32 + lane] = acc[0];
  if (__syncthreads_and(ok ? 1 : 0) == 0) return false;
  // CTA reduction in warp order, one partial per (tile, CTA)
  const int c0 = p_range_lo(U, x.cta, x.grid), c1 = p_range_lo(U, x.cta + 1, x.grid);
  if (c1 > c0) {
    const int t0 = c0 / B, t1 = (c1 - 1) / B;
    const float* redall = reinterpret_cast<const float*>(smem + SM_RED);
    for (int idx = threadIdx.x; idx < (t1 - t0 + 1) * 32; idx += blockDim.x) {
      const int t = t0 + idx / 32, row = idx & 31;
      float s = 0.0f;
      for (int w = 0; w < P_WARPS; ++w) {
        const int a = wt[2 * w], n = wt[2 * w + 1];
        if (n > 0 && t >= a && t < a + n) s += redall[(w * P_WARP_TILES + (t - a)) * 32 + row];
      }
      const int seg = x.cta - p_cta_of(t * B, U, x.grid);
      part[(size_t(t) * maxseg + seg) * 32 + row] = s;
    }
  }
  return true;
}

// ---- attention stage ---------------------------------------------------------------------

// NV f64 sums over the CTA at once (two barriers).
template <int NV>
__device__ __forceinline__ void block_sums(double (&v)[NV], double* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < NV; ++k) v[k] = warp_sum_d(v[k]);
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < NV; ++k) scratch[warp * NV + k] = v[k];
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    double t = 0.0;
    for (int w = 0; w < P_WARPS; ++w) t += scratch[w * NV + k];
    v[k] = t;
  }
  __syncthreads();
}

__device__ __forceinline__ void combine_kvh(const StreamCtx& x, int kvh, uint8_t* smem);

__device__ __forceinline__ bool attention_stage(const StreamCtx& x, Ring& r, int l, uint8_t* smem) {
  const PParams& p = *x.p;
  const PLayer& L = p.layers[l];
  const int G = p.H / p.KVH, KVH = p.KVH;
  const int kvh = x.cta / x.att_cpk, j = x.cta % x.att_cpk;
  const bool active = kvh < KVH;
  const int pos = p.pos[0];
  const int nu = (x.count + P_ATT_TOK - 1) / P_ATT_TOK;
  const int u0 = active ? p_range_lo(nu, j, x.att_cpk) : 0, u1 = active ? p_range_lo(nu, j + 1, x.att_cpk) : 0;
  const bool has_fresh = active && pos >= u0 * P_ATT_TOK && pos < u1 * P_ATT_TOK;
  float* qs = reinterpret_cast<float*>(smem + SM_QS);
  float* fk = reinterpret_cast<float*>(smem + SM_FRESH);
  float* fv = fk + 256;
  double* scratch = reinterpret_cast<double*>(smem + SM_MISC);
  const int d = threadIdx.x;
  if (active) {
    // Vectors of this KV head (thread d = dimension): the G query heads and,
    // for the CTA that holds the new token of an own-KV layer, its key and
    // value.  QK-norm (f64 sums) and NeoX RoPE as head_norm_rope of the per-kernel step; queries
    // are rounded with the Rust f16 codec (lib.rs:590-597).
    constexpr int NV = P_MAX_G + 2;
    const bool fresh_own = has_fresh && L.own_kv;
    const int qrows = p.H * 256, kvrows = KVH * 256;
    int rows[NV];
#pragma unroll
    for (int g = 0; g < P_MAX_G; ++g) rows[g] = g < G ? (kvh * G + g) * 256 + d : -1;
    rows[P_MAX_G] = fresh_own ? qrows + kvh * 256 + d : -1;
    rows[P_MAX_G + 1] = fresh_own ? qrows + kvrows + kvh * 256 + d : -1;
    float v[NV];
    gemv_rows<NV>(L.qkv, rows, x.grid, v);
    double ss[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) ss[k] = double(v[k]) * double(v[k]);
    block_sums<NV>(ss, scratch);
    const double wq = double(__ldg(L.n_q + d)), wk = double(__ldg(L.n_k + d));
    float* nb = reinterpret_cast<float*>(smem + SM_ACT);  // [NV][256]
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const double sc = 1.0 / sqrt(ss[k] / 256.0 + p.eps);
      const float n = k < P_MAX_G ? float((double(v[k]) * sc) * wq)
                                  : (k == P_MAX_G ? float((double(v[k]) * sc) * wk) : float(double(v[k]) * sc));
      nb[k * 256 + d] = n;
    }
    __syncthreads();
    const int idx = d & 127;
    const double c = p.cos_t[idx], sn = p.sin_t[idx];
    float rot[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const float a = nb[k * 256 + (d & 127)], b = nb[k * 256 + 128 + (d & 127)];
      rot[k] = d < 128 ? float(double(a) * c) - float(double(b) * sn) : float(double(a) * sn) + float(double(b) * c);
    }
#pragma unroll
    for (int g = 0; g < P_MAX_G; ++g)
      if (g < G) qs[g * 256 + d] = round_f16_rust(rot[g]);
    if (has_fresh) {
      const size_t row = (size_t(pos) * KVH + kvh) * 256 + d;
      if (fresh_own) {
        const float kn = rot[P_MAX_G], vn = nb[(P_MAX_G + 1) * 256 + d];
        fk[d] = kn;
        fv[d] = vn;
        L.kc[row] = kn;
        L.vc[row] = vn;
      } else {
        fk[d] = __ldcg(L.kc + row);
        fv[d] = __ldcg(L.vc + row);
      }
    }
  }
  __syncthreads();
  // units: warps < P_ATT_WARPS, lane owns dims lane + 32 i
  const int warp = x.warp, lane = x.lane;
  bool ok = true;
  float* stagep = reinterpret_cast<float*>(smem + SM_ACT) + warp * P_ATT_REC;
  if (warp < P_ATT_WARPS) {
    int lo, hi;
    warp_range(x, l, ST_ATT, &lo, &hi);
    float q[P_MAX_G][8], o[P_MAX_G][8], mrun[P_MAX_G], lrun[P_MAX_G];
#pragma unroll
    for (int g = 0; g < P_MAX_G; ++g) {
      mrun[g] = -INFINITY;
      lrun[g] = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        q[g][i] = g < G ? qs[g * 256 + lane + 32 * i] : 0.0f;
        o[g][i] = 0.0f;
      }
    }
#pragma unroll 1
    for (int u = lo; u < hi; ++u) {
      if (!ring_wait(p, r)) {
        ok = false;
        break;
      }
      const float* K = reinterpret_cast<const float*>(ring_slot(r, r.seq));
      const float* V = K + P_ATT_TOK * 256;
      const int t0 = u * P_ATT_TOK;
      // scores s[g][t], reduced so that lane L ends with value k = L >> 1 (k = g*4 + t)
      float s[16];
      const int fresh_t = has_fresh ? pos - t0 : -1;  // token of this unit that is the new row, if any
#pragma unroll
      for (int t = 0; t < P_ATT_TOK; ++t) {
        const float* kr = (t == fresh_t) ? fk : K + t * 256;
        float kd[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) kd[i] = kr[lane + 32 * i];
#pragma unroll
        for (int g = 0; g < P_MAX_G; ++g) {
          float a = 0.0f;
#pragma unroll
          for (int i = 0; i < 8; ++i) a = fmaf(q[g][i], kd[i], a);
          s[g * 4 + t] = a;
        }
      }
      // reduce-scatter: after offsets 16, 8, 4, 2 lane L holds partial sums of value L >> 1
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const bool up = lane & 16;
        const float send = up ? s[k] : s[k + 8];
        const float keep = up ? s[k + 8] : s[k];
        s[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const bool up = lane & 8;
        const float send = up ? s[k] : s[k + 4];
        const float keep = up ? s[k + 4] : s[k];
        s[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const bool up = lane & 4;
        const float send = up ? s[k] : s[k + 2];
        const float keep = up ? s[k + 2] : s[k];
        s[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
      {
        const bool up = lane & 2;
        const float send = up ? s[0] : s[1];
        const float keep = up ? s[1] : s[0];
        s[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
      }
      s[0] += __shfl_xor_sync(0xffffffffu, s[0], 1);
      // lane L: value k = L >> 1, head g = L >> 3, token t = (L >> 1) & 3
      const int kg = lane >> 3, kt = (lane >> 1) & 3;
      const bool valid = (t0 + kt) < x.count;
      const float sc = valid ? s[0] : -INFINITY;
      float mx = sc;
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      // running max of head kg (every lane keeps every head's state)
      float mold = mrun[0];
#pragma unroll
      for (int g = 1; g < P_MAX_G; ++g)
        if (kg == g) mold = mrun[g];
      const float mnew = fmaxf(mold, mx);
      const float pk = (sc == -INFINITY) ? 0.0f : float(exp(double(sc - mnew)));
      const float corr = (mold == -INFINITY) ? 0.0f : float(exp(double(mold - mnew)));
#pragma unroll
      for (int g = 0; g < P_MAX_G; ++g) {
        const float cg = __shfl_sync(0xffffffffu, corr, 8 * g);
        const float mg = __shfl_sync(0xffffffffu, mnew, 8 * g);
        float pg[P_ATT_TOK], psum = 0.0f;
#pragma unroll
        for (int t = 0; t < P_ATT_TOK; ++t) {
          pg[t] = __shfl_sync(0xffffffffu, pk, 8 * g + 2 * t);
          psum += pg[t];
        }
        if (g < G) {
          lrun[g] = lrun[g] * cg + psum;
          mrun[g] = mg;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float a = o[g][i] * cg;
#pragma unroll
            for (int t = 0; t < P_ATT_TOK; ++t) {
              const float* vr = (t == fresh_t) ? fv : V + t * 256;
              a = fmaf(pg[t], vr[lane + 32 * i], a);
            }
            o[g][i] = a;
          }
        }
      }
      ring_release(x, r);
    }
    // stage this warp's partial (m, l, o) for the CTA merge
#pragma unroll
    for (int g = 0; g < P_MAX_G; ++g) {
      if (lane == 0) {
        stagep[g] = mrun[g];
        stagep[P_MAX_G + g] = lrun[g];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) stagep[2 * P_MAX_G + g * 256 + lane + 32 * i] = o[g][i];
    }
  }
  if (__syncthreads_and(ok ? 1 : 0) == 0) return false;
  // merge the attention warps' partials (d = thread = dimension)
  if (active) {
    float* out = p.att_part + size_t(x.cta) * P_ATT_REC;
    const float* st0 = reinterpret_cast<const float*>(smem + SM_ACT);
    for (int g = 0; g < G; ++g) {
      float M = -INFINITY;
      for (int w = 0; w < P_ATT_WARPS; ++w) M = fmaxf(M, st0[w * P_ATT_REC + g]);
      float lsum = 0.0f, osum = 0.0f;
      for (int w = 0; w < P_ATT_WARPS; ++w) {
        const float mw = st0[w * P_ATT_REC + g];
        const float wt = (mw == -INFINITY) ? 0.0f : float(exp(double(mw - M)));
        lsum += wt * st0[w * P_ATT_REC + P_MAX_G + g];
        osum += wt * st0[w * P_ATT_REC + 2 * P_MAX_G + g * 256 + d];
      }
      if (d == 0) {
        out[g] = M;
        out[P_MAX_G + g] = lsum;
      }
      out[2 * P_MAX_G + g * 256 + d] = osum;
    }
  }
  // The last attention CTA of this KV head merges the head group.
  int* flag = reinterpret_cast<int*>(smem + SM_MISC + 320);
  __syncthreads();
  if (threadIdx.x == 0) {
    int last = 0;
    if (active) {
      __threadfence();
      const unsigned old = atomicAdd(p.kvh_counters + size_t(l) * KVH + kvh, 1u);
      last = int(old) + 1 == x.att_cpk;
      __threadfence();
    }
    *flag = last;
  }
  __syncthreads();
  if (*flag) {
    combine_kvh(x, kvh, smem);
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      atomicAdd(counter(p, l, PS_COMB), 1u);
    }
  }
  return true;
}

// Merges the per-CTA attention partials of the G query heads of KV head kvh
// (attn_combine_kernel arithmetic: global max, f64-exp weights, f64
// normalizer, weighted sum in CTA order), casts through the TS f16 codec and
// quantizes Q8_K blocks kvh*G .. kvh*G+G-1 of the O projection's input.
// Run by the last attention CTA of the KV head.
__device__ __forceinline__ void combine_kvh(const StreamCtx& x, int kvh, uint8_t* smem) {
  const PParams& p = *x.p;
  const int G = p.H / p.KVH, nc = x.att_cpk, d = threadIdx.x, lane = x.lane, warp = x.warp;
  float* wch = reinterpret_cast<float*>(smem + SM_QS);  // [P_MAX_G][256] weights
  double* lsum = reinterpret_cast<double*>(smem + SM_MISC);  // [P_MAX_G]
  float* vec = reinterpret_cast<float*>(smem + SM_ACT);  // [P_MAX_G][256]
  const float* base = p.att_part + size_t(kvh * nc) * P_ATT_REC;
  if (warp < G) {
    const int g = warp;
    float mx = -INFINITY;
    for (int j = lane; j < nc; j += 32) mx = fmaxf(mx, __ldcg(base + size_t(j) * P_ATT_REC + g));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    double lw = 0.0;
    for (int j = lane; j < nc; j += 32) {
      const float mc = __ldcg(base + size_t(j) * P_ATT_REC + g);
      const float w = mc == -INFINITY ? 0.0f : float(exp(double(mc - mx)));
      wch[g * 256 + j] = w;
      lw += double(w) * double(__ldcg(base + size_t(j) * P_ATT_REC + P_MAX_G + g));
    }
    lw = warp_sum_d(lw);
    if (lane == 0) lsum[g] = lw;
  }
  __syncthreads();
  // thread (g, q): dimensions 4q..4q+3 of head g; 16 float4 loads in flight,
  // unconditional (record index clamped, its weight zero beyond nc)
  {
    const int g = threadIdx.x >> 6, q = threadIdx.x & 63;
    if (g < G) {
      const float4* po = reinterpret_cast<const float4*>(base + 2 * P_MAX_G + g * 256) + q;
      constexpr int R4 = P_ATT_REC / 4;  // float4 per record
      float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int c = 0; c < nc; c += 16) {
        float4 v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = __ldcg(po + size_t(min(c + i, nc - 1)) * R4);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float w = c + i < nc ? wch[g * 256 + c + i] : 0.0f;
          o4.x += w * v[i].x;
          o4.y += w * v[i].y;
          o4.z += w * v[i].z;
          o4.w += w * v[i].w;
        }
      }
      const double L = lsum[g];
      vec[g * 256 + 4 * q + 0] = round_f16_ts(float(double(o4.x) / L));
      vec[g * 256 + 4 * q + 1] = round_f16_ts(float(double(o4.y) / L));
      vec[g * 256 + 4 * q + 2] = round_f16_ts(float(double(o4.z) / L));
      vec[g * 256 + 4 * q + 3] = round_f16_ts(float(double(o4.w) / L));
    }
  }
  __syncthreads();
  if (warp < G) {
    const int h = kvh * G + warp, nb = p.H;
    float v8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v8[i] = vec[warp * 256 + 8 * lane + i];
    q8k_block_warp(v8, lane, smem + SM_STAGE + warp * 256, p.q8_attn + size_t(h) * Q8A_REC,
                   p.q8_attn + ((size_t(nb) * Q8A_REC + 255) & ~size_t(255)) + size_t(h) * Q8B_REC);
  }
}

// One warp: GEGLU of 256-block b of the FFN activation and its Q8_K records
// (geglu_quant_kernel arithmetic).  `scratch` is 256 floats of this warp's
// shared memory (the loop over the f64 tanh is not unrolled, to keep code
// small).
__device__ __forceinline__ void geglu_block(const StreamCtx& x, const PLayer& L, int b, float* scratch,
                                            uint8_t* stage) {
  const PParams& p = *x.p;
  const int lane = x.lane, F = p.F;
  float gu[16];
  const int e0 = b * 256 + 8 * lane;
  int rows[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    rows[i] = e0 + i;
    rows[8 + i] = F + e0 + i;
  }
  gemv_rows<16>(L.gu, rows, x.grid, gu);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    scratch[8 * lane + i] = gu[i];
    scratch[8 * lane + i + 256] = gu[8 + i];
  }
  __syncwarp();
#pragma unroll 1
  for (int i = 0; i < 8; ++i) {
    const float g = scratch[8 * lane + i], u = scratch[256 + 8 * lane + i];
    scratch[8 * lane + i] = float(gelu_ts(g) * double(u));
  }
  __syncwarp();
  float a[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = scratch[8 * lane + i];
  const int nb = F / 256;
  q8k_block_warp(a, lane, stage, p.q8_act + size_t(b) * Q8A_REC,
                 p.q8_act + ((size_t(nb) * Q8A_REC + 255) & ~size_t(255)) + size_t(b) * Q8B_REC);
}

// After this CTA's gate/up partials are stored: it counts itself in every
// 256-block of the activation whose gate or up tiles it produced; the CTA
// that completes a block (the last of its producers) computes that block's
// GEGLU + Q8_K at once, and adds the blocks it finished to the ACT counter.
// The activation is thus built by up to F/256 CTAs as soon as each block's
// inputs exist, without a separate stage.
__device__ __forceinline__ void gu_epilogue(const StreamCtx& x, const PLayer& L, int l, uint8_t* smem) {
  const PParams& p = *x.p;
  const PGemv& g = L.gu;
  const int B = pl_i(g.B), U = pl_i(g.tiles) * B, half = p.F / 32;  // tiles of the gate part
  int* mine = reinterpret_cast<int*>(smem + SM_MISC + 320);          // [0] = count, [1..16] = blocks
  unsigned* bc = p.blk_counters + size_t(l) * (p.F / 256);
  __syncthreads();  // the CTA's partials are stored
  if (threadIdx.x == 0) {
    __threadfence();
    int n = 0;
    const int c0 = p_range_lo(U, x.cta, x.grid), c1 = p_range_lo(U, x.cta + 1, x.grid);
    if (c1 > c0) {
      const int t0 = c0 / B, t1 = (c1 - 1) / B;
      for (int part = 0; part < 2; ++part) {
        const int lo = max(t0, part * half), hi = min(t1, part * half + half - 1);
        for (int blk = (lo - part * half) / 8; lo <= hi && blk <= (hi - part * half) / 8; ++blk) {
          int target = 0;
          for (int q = 0; q < 2; ++q) {
            const int ta = q * half + 8 * blk, tb = ta + 7;
            target += p_cta_of(tb * B + B - 1, U, x.grid) - p_cta_of(ta * B, U, x.grid) + 1;
          }
          const unsigned old = atomicAdd(bc + blk, 1u);
          if (int(old) + 1 == target && n < 16) mine[1 + n++] = blk;
        }
      }
    }
    mine[0] = n;
    __threadfence();
  }
  __syncthreads();
  const int n = mine[0];
  float* scratch = reinterpret_cast<float*>(smem + SM_ACT) + x.warp * 512;
  for (int i = x.warp; i < n; i += P_WARPS)
    geglu_block(x, L, mine[1 + i], scratch, smem + SM_STAGE + x.warp * 256);
  __syncthreads();
  if (threadIdx.x == 0 && n > 0) {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __threadfence();
    atomicAdd(counter(p, l, PS_ACT), unsigned(n));
  }
}

// The hidden size is 2048 (one 256-block per warp); checked on the host.
__device__ __forceinline__ void prologue_attn(const PParams& p, int l, uint8_t* smem, int grid) {
  prologue_attn_input<1>(p, l, smem, grid);
}

// The hidden size is 2048 (one 256-block per warp); checked on the host.
__device__ __forceinline__ void prologue_ffn(const PParams& p, int l, uint8_t* smem, int grid) {
  prologue_ffn_input<1>(p, l, smem, grid);
}

// CTA 0 after the last layer: x_L = H1 + rmsnorm(down_{L-1}) * w_post_ffw.
template <int NBW>
__device__ __forceinline__ void final_residual(const PParams& p, const StreamCtx& x, uint8_t* smem) {
  const int l = p.nlayers - 1;
  const PLayer& L = p.layers[l];
  const int D = p.D;
  float y[NBW][8];
#pragma unroll
  for (int j = 0; j < NBW; ++j) gemv_rows8(L.down, (x.warp + P_WARPS * j) * 256 + 8 * x.lane, x.grid, y[j]);
  const double sc = block_rms_scale<NBW>(y, NBW, D, p.eps, reinterpret_cast<double*>(smem + SM_MISC));
#pragma unroll
  for (int j = 0; j < NBW; ++j) {
    const int e0 = (x.warp + P_WARPS * j) * 256 + 8 * x.lane;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      p.X[e0 + i] = __ldcg(p.H1 + e0 + i) + float((double(y[j][i]) * sc) * double(__ldg(L.n_post_ffw + e0 + i)));
  }
}

}  // namespace

__global__ void __launch_bounds__(P_THREADS, 1) persistent_step_kernel(const PParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  StreamCtx x;
  x.p = &p;
  x.grid = gridDim.x;
  x.cta = blockIdx.x;
  x.warp = threadIdx.x >> 5;
  x.lane = threadIdx.x & 31;
  x.count = min(p.cap, p.pos[0] + 1);
  x.att_cpk = gridDim.x / p.KVH;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM_BARS);
  if (x.lane == 0) {
    for (int s = 0; s < P_SLOTS; ++s) mbar_init(bars + x.warp * P_SLOTS + s, 1);
  }
  __syncwarp();
  Ring r;
  r.base = smem + SM_RING + size_t(x.warp) * P_SLOTS * P_SLOT_BYTES;
  r.bars = bars + x.warp * P_SLOTS;
  r.seq = r.issued = 0;
  r.issue = cursor_begin(x);
  ring_fill(x, r);
  __syncthreads();

  const unsigned grid = gridDim.x;
  const int act_blocks = p.F / 256;
  bool ok = true;
  // One pass of the stage driver per (layer, stage): every stage body has a
  // single call site, so the kernel's code stays small enough for the
  // instruction caches while each layer sweeps through it.
#pragma unroll 1
  for (int l = 0; l < p.nlayers && ok; ++l) {
    const PLayer& L = p.layers[l];
#pragma unroll 1
    for (int st = 0; st < PS_COUNT && ok; ++st) {
      // 1. wait for the producers of this stage's input
      const unsigned* dep = nullptr;
      unsigned need = grid;
      bool runs = true;  // does this CTA take part in the stage?
      switch (st) {
        case PS_QKV: dep = l > 0 ? counter(p, l - 1, PS_DOWN) : nullptr; break;
        case PS_ATT: dep = counter(p, l, PS_QKV); break;
        case PS_COMB: runs = false; break;  // done by the last attention CTA of each KV head
        case PS_O: dep = counter(p, l, PS_COMB); need = unsigned(p.KVH); break;
        case PS_GU: dep = counter(p, l, PS_O); break;
        case PS_ACT: runs = false; break;  // done by the last producer of each activation block
        default: dep = counter(p, l, PS_ACT); need = unsigned(act_blocks); break;
      }
      if (!runs) continue;
      if (dep && !(ok = cta_wait(p, dep, need))) break;
      // 2. stage the input (prologue or records written by other CTAs)
      if (st == PS_QKV) {
        prologue_attn(p, l, smem, grid);
      } else if (st == PS_O) {
        const int nb = p.H;
        stage_records(smem + SM_ACT, p.q8_attn, nb * Q8A_REC);
        stage_records(smem + SM_ACT + nb * Q8A_REC, p.q8_attn + ((size_t(nb) * Q8A_REC + 255) & ~size_t(255)),
                      nb * Q8B_REC);
      } else if (st == PS_GU) {
        prologue_ffn(p, l, smem, grid);
      } else if (st == PS_DOWN) {
        const int nb = p.F / 256;
        const bool q6 = pl_i(L.down.type[0]) == TYPE_Q6_K;
        const uint8_t* src = q6 ? p.q8_act + ((size_t(nb) * Q8A_REC + 255) & ~size_t(255)) : p.q8_act;
        stage_records(smem + SM_ACT, src, nb * (q6 ? Q8B_REC : Q8A_REC));
      }
      __syncthreads();
      // 3. the stage's work
      if (st == PS_ATT) {
        ok = attention_stage(x, r, l, smem);
      } else {
        const PGemv& g = st == PS_QKV ? L.qkv : (st == PS_O ? L.o : (st == PS_GU ? L.gu : L.down));
        ok = gemv_stage(x, r, g, smem, st == PS_DOWN);
      }
      if (!ok) break;
      // 4. publish
      if (st == PS_GU) gu_epilogue(x, L, l, smem);
      else cta_signal(counter(p, l, st));
    }
  }
  if (!ok) {
    if (threadIdx.x == 0) atomicExch(p.abort_word, 1);
    ring_drain(p, r);
    return;
  }
  // final residual x_L = H1 + rmsnorm(down_{L-1}) * w_post_ffw (CTA 0)
  if (x.cta == 0) {
    const int l = p.nlayers - 1;
    if (!cta_wait(p, counter(p, l, PS_DOWN), grid)) {
      ring_drain(p, r);
      return;
    }
    final_residual<1>(p, x, smem);
  }
}

size_t persist_smem_bytes() { return SM_TOTAL; }

int persist_maxseg(int tiles, int B, int grid, bool* warp_tiles_ok) {
  const int U = tiles * B;
  int mx = 1;
  for (int t = 0; t < tiles; ++t) {
    const int n = p_cta_of(t * B + B - 1, U, grid) - p_cta_of(t * B, U, grid) + 1;
    if (n > mx) mx = n;
  }
  bool ok = true;
  for (int c = 0; c < grid && ok; ++c) {
    const int c0 = p_range_lo(U, c, grid), c1 = p_range_lo(U, c + 1, grid), n = c1 - c0;
    for (int w = 0; w < P_WARPS; ++w) {
      const int lo = c0 + n * w / P_WARPS, hi = c0 + n * (w + 1) / P_WARPS;
      if (hi > lo && (hi - 1) / B - lo / B + 1 > P_WARP_TILES) ok = false;
    }
  }
  if (warp_tiles_ok) *warp_tiles_ok = ok;
  return mx;
}

int persist_grid() {
  // per device: the grid + 1 once computed, 0 before (a failed query is not
  // kept, so the next call asks again)
  static std::atomic<int> cached[64];
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  const int c = cached[dev].load(std::memory_order_acquire);
  if (c > 0) return c - 1;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (cudaFuncSetAttribute(persistent_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(SM_TOTAL)) !=
      cudaSuccess)
    return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, persistent_step_kernel, P_THREADS, SM_TOTAL) !=
      cudaSuccess)
    return 0;
  const int grid = per_sm >= 1 ? sms : 0;
  cached[dev].store(grid + 1, std::memory_order_release);
  return grid;
}

cudaError_t launch_persistent_step(const PParams& p, int grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(P_THREADS);
  cfg.dynamicSmemBytes = SM_TOTAL;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, persistent_step_kernel, p);
}

}  // namespace hc
