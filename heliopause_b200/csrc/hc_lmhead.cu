// hc_lmhead.cu -- vocabulary LM head fused with top-k candidate selection.
//
// Replaces the reference's output path:
//   WASM   : forwardOutput (runner/wasm/layers.ts:381-416) materializes all
//            262,144 logits, applies the softcap, then topK (runtime.ts:514)
//   WebGPU : dispatchOutputTopK (runner/webgpu/segment-runner.ts:3208-3248):
//            per-stripe GEMV into scratch logits, chunked top-k
//            (TOPK_CHUNK_CANDIDATES_WGSL, shaders.ts:1591) and a merge
//            (TOPK_MERGE_CANDIDATES_WGSL, shaders.ts:1652); the softcap is
//            applied to the k survivors on the host (mergeTopCandidates,
//            segment-runner.ts:3773-3794).
// Here the logits never reach HBM: a persistent grid walks the 32-row tiles,
// each CTA keeps a running top-k per column in shared memory, and a second
// kernel merges the per-CTA lists by radix selection.
//
// Ordering: value descending, then id ascending -- the tie rule of both
// reference paths (runtime.ts:514-527 keeps the earlier id; the WGSL
// betterValue() compares ids).  It is encoded in one 64-bit key
//   key = orderable(value) << 32 | (0xFFFFFFFF - id)
// so larger key = better candidate, every key is distinct, -0 == +0, and NaN
// ranks below every number.  Key 0 is the empty-slot sentinel.
#include "hc_common.cuh"
#include "hc_gemv_body.cuh"
#include "hc_kernels.cuh"
#include "hc_lmhead.cuh"
#include "hc_mma_stream.cuh"

namespace hc {

__device__ __forceinline__ uint64_t topk_key(float v, uint32_t id) {
  uint32_t b = __float_as_uint(v);
  if (v == 0.0f) b = 0;  // -0 ranks with +0
  uint32_t ord = (v != v) ? 0u : ((b & 0x80000000u) ? ~b : (b | 0x80000000u));
  return (uint64_t(ord) << 32) | uint64_t(0xffffffffu - id);
}

__device__ __forceinline__ void topk_decode(uint64_t key, int32_t* id, float* v) {
  const uint32_t ord = uint32_t(key >> 32);
  const uint32_t b = (ord & 0x80000000u) ? (ord & 0x7fffffffu) : ~ord;
  *v = __uint_as_float(b);
  *id = int32_t(0xffffffffu - uint32_t(key));
}

// Warp-cooperative insertion of each lane's key into a descending list of k
// (<= 64) keys held in shared memory.  Only keys above the current k-th entry
// are inserted, one at a time in lane order, so the list stays exact.
__device__ __forceinline__ void topk_insert_warp(uint64_t* list, int k, uint64_t key, int lane) {
  uint64_t thr = list[k - 1];
  unsigned mask = __ballot_sync(0xffffffffu, key > thr);
  while (mask) {
    const int src = __ffs(mask) - 1;
    const uint64_t x = __shfl_sync(0xffffffffu, key, src);
    const uint64_t a = lane < k ? list[lane] : 0ull;
    const uint64_t b = lane + 32 < k ? list[lane + 32] : 0ull;
    const int pos = __popc(__ballot_sync(0xffffffffu, lane < k && a > x)) +
                    __popc(__ballot_sync(0xffffffffu, lane + 32 < k && b > x));
    const uint64_t a_prev = __shfl_up_sync(0xffffffffu, a, 1);
    const uint64_t b_prev = __shfl_up_sync(0xffffffffu, b, 1);
    const uint64_t a31 = __shfl_sync(0xffffffffu, a, 31);
    const uint64_t na = lane < pos ? a : (lane == pos ? x : a_prev);
    const int ib = lane + 32;
    const uint64_t nb = ib < pos ? b : (ib == pos ? x : (lane == 0 ? a31 : b_prev));
    __syncwarp();
    if (lane < k) list[lane] = na;
    if (ib < k) list[ib] = nb;
    __syncwarp();
    thr = list[k - 1];
    mask &= ~(1u << src);
    mask &= __ballot_sync(0xffffffffu, key > thr);
  }
}

// Flush of the LM head: insert the tile's logits into this warp's lists.
template <int NC>
struct TopkFlush {
  const LmHeadParams* P;
  uint64_t* best;  // [NC][TOPK_MAX] of the calling warp
  int lane;
  __device__ __forceinline__ void operator()(int tile, const float (&v)[NC]) {
    const int row = tile * TILE + lane;
    const int rows = P->g.seg[0].rows;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      if (c < P->g.ncols) {
        const uint64_t key = row < rows ? topk_key(v[c], uint32_t(P->id_offset + row)) : 0ull;
        topk_insert_warp(best + c * TOPK_MAX, P->k, key, lane);
      }
    }
  }
};

// Persistent grid over the head's tiles; every warp owns whole tiles and its
// own running top-k per column, so no barrier is needed until the end.
template <int NC>
__global__ void __launch_bounds__(GEMV_THREADS, GEMV_CTAS_PER_SM) hc_lmhead_topk_kernel(
    const __grid_constant__ LmHeadParams P) {
  const GemvParams& p = P.g;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ uint64_t best[GEMV_WARPS_PER_CTA][NC][TOPK_MAX];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.launch_dependents;");
#endif
  const int nitems = p.total_tiles;
  const int item0 = blockIdx.x * GEMV_WARPS_PER_CTA + warp, istride = gridDim.x * GEMV_WARPS_PER_CTA;
  UnitRegs buf[2];
  int first_type = TYPE_Q4_K;
  if (item0 < nitems) load_unit(buf[0], unit_addr(p, item0, 0, &first_type), first_type, lane);
  for (int i = threadIdx.x; i < GEMV_WARPS_PER_CTA * NC * TOPK_MAX; i += blockDim.x) (&best[0][0][0])[i] = 0ull;
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
  bool need_a, need_b;
  gemv_planes(p, &need_a, &need_b);
  uint8_t* act_a = need_a ? smem : nullptr;
  uint8_t* act_b = need_b ? smem + (need_a ? size_t(p.ncols) * p.nb * Q8A_REC : 0) : nullptr;
  stage_activations(p, act_a, act_b, 0, p.nb);
  __syncthreads();
  const ActSlice act{act_a, act_b, p.nb, 0};
  TopkFlush<NC> flush{&P, &best[warp][0][0], lane};
  // whole tiles per warp, blocks in order: the reference's f32 order per row
  stream_items<NC, UNIT_CHUNKS, true>(p, act, item0, istride, nitems, lane, buf[0], first_type, flush);
  __syncthreads();
  // Merge the four warp lists into this CTA's top-k: a real key's rank is its
  // index in its own list plus, for each other list, the number of larger
  // keys there (binary search; real keys are distinct, empty slots are 0).
  for (int c = 0; c < p.ncols; ++c) {
    uint64_t* out = P.cand + size_t(p.col0 + c) * P.cand_col_stride + size_t(blockIdx.x) * P.k;
    for (int i = threadIdx.x; i < P.k; i += blockDim.x) out[i] = 0ull;
  }
  __syncthreads();
  for (int c = 0; c < p.ncols; ++c) {
    uint64_t* out = P.cand + size_t(p.col0 + c) * P.cand_col_stride + size_t(blockIdx.x) * P.k;
    for (int t = threadIdx.x; t < GEMV_WARPS_PER_CTA * P.k; t += blockDim.x) {
      const int w = t / P.k, i = t % P.k;
      const uint64_t e = best[w][c][i];
      if (e == 0ull) continue;
      int rank = i;
      for (int o = 0; o < GEMV_WARPS_PER_CTA; ++o) {
        if (o == w) continue;
        int lo = 0, hi = P.k;  // first index whose key is <= e
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (best[o][c][mid] > e) lo = mid + 1;
          else hi = mid;
        }
        rank += lo;
      }
      if (rank < P.k) out[rank] = e;
    }
  }
}

// Tensor-core LM head for 3..8 columns: the weight stream and block products
// of the tensor-core GEMV (hc_mma_stream.cuh) over a persistent grid of
// LMM_WARPS-warp CTAs walking the head's tiles, fused with the same per-warp
// top-k lists as hc_lmhead_topk_kernel.  A finished tile's 32 x 8 sums go from
// the accumulator layout to lane = row through a padded shared-memory
// transpose, then each column's keys are inserted into the warp's list.  The
// CTA merges its warps' lists by rank into k candidates per column at
// cand[col * cand_col_stride + blockIdx.x * k].
constexpr int LMM_WARPS = 8;
constexpr int LMM_TSTRIDE = 36;  // transpose row stride: conflict-free writes (accumulator layout) and reads

__host__ __device__ inline size_t lmm_list_bytes(const LmHeadParams& P) {
  return size_t(LMM_WARPS) * P.g.ncols * P.k * sizeof(uint64_t);
}

__global__ void __launch_bounds__(LMM_WARPS * 32, 1) hc_lmhead_mma_kernel(const __grid_constant__ LmHeadParams P) {
  const GemvParams& p = P.g;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float tr[LMM_WARPS][GM_COLS * LMM_TSTRIDE];
  __shared__ __align__(8) uint64_t bars[LMM_WARPS][4];
  __shared__ __align__(8) uint64_t act_bar;
  const int lane = int(threadIdx.x & 31), warp = int(threadIdx.x >> 5), g = lane >> 2, t = lane & 3;
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.launch_dependents;");
#endif
  const int nitems = p.total_tiles;
  const int item0 = int(blockIdx.x) * LMM_WARPS + warp, istride = int(gridDim.x) * LMM_WARPS;
  bool need_a, need_b;
  gemv_planes(p, &need_a, &need_b);
  const int cs_a = gm_col_stride(p.nb, Q8A_REC), cs_b = gm_col_stride(p.nb, Q8B_REC);
  uint8_t* act_a = need_a ? smem : nullptr;
  uint8_t* act_b = need_b ? smem + (need_a ? size_t(GM_COLS) * cs_a : 0) : nullptr;
  uint64_t* lists = reinterpret_cast<uint64_t*>(smem + gm_act_bytes(p, p.nb));  // [warp][col][k]
  const int slot = gm_slot_bytes(p);
  uint8_t* ring = smem + gm_act_bytes(p, p.nb) + (lmm_list_bytes(P) + 15) / 16 * 16;
  MmaStream ms(p, item0, istride, nitems, ring + size_t(warp) * p.ring * slot, slot, bars[warp], lane);
  ms.prime();
  const int nl = LMM_WARPS * p.ncols * P.k;
  for (int i = int(threadIdx.x); i < nl; i += int(blockDim.x)) lists[i] = 0ull;
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
  stage_act_slice8(p, act_a, act_b, cs_a, cs_b, 0, p.nb, &act_bar);
  __syncthreads();
  bool ok = mbar_wait_parity(&act_bar, 0, p.err);
  float* trw = tr[warp];
  uint64_t* wl = lists + size_t(warp) * p.ncols * P.k;
  const int rows = p.seg[0].rows;
  auto flush = [&](int tile, const float (&acc)[2][1][4]) {
#pragma unroll
    for (int mg = 0; mg < 2; ++mg)
#pragma unroll
      for (int r = 0; r < 4; ++r) trw[(2 * t + (r & 1)) * LMM_TSTRIDE + 16 * mg + g + 8 * (r >> 1)] = acc[mg][0][r];
    __syncwarp();
    const int row = tile * TILE + lane;
    for (int c = 0; c < p.ncols; ++c) {
      const uint64_t key = row < rows ? topk_key(trw[c * LMM_TSTRIDE + lane], uint32_t(P.id_offset + row)) : 0ull;
      topk_insert_warp(wl + c * P.k, P.k, key, lane);
    }
    __syncwarp();
  };
  ms.run(act_a, act_b, cs_a, cs_b, 0, ok, g, t, flush);
  __syncthreads();
  // merge the warps' lists by rank (real keys are distinct; empty slots are 0)
  for (int c = 0; c < p.ncols; ++c) {
    uint64_t* out = P.cand + size_t(p.col0 + c) * P.cand_col_stride + size_t(blockIdx.x) * P.k;
    for (int i = int(threadIdx.x); i < P.k; i += int(blockDim.x)) out[i] = 0ull;
  }
  __syncthreads();
  for (int c = 0; c < p.ncols; ++c) {
    uint64_t* out = P.cand + size_t(p.col0 + c) * P.cand_col_stride + size_t(blockIdx.x) * P.k;
    for (int x = int(threadIdx.x); x < LMM_WARPS * P.k; x += int(blockDim.x)) {
      const int w = x / P.k, i = x % P.k;
      const uint64_t e = lists[(size_t(w) * p.ncols + c) * P.k + i];
      if (e == 0ull) continue;
      int rank = i;
      for (int o = 0; o < LMM_WARPS; ++o) {
        if (o == w) continue;
        const uint64_t* lo_list = lists + (size_t(o) * p.ncols + c) * P.k;
        int lo = 0, hi = P.k;  // first index whose key is <= e
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (lo_list[mid] > e) lo = mid + 1;
          else hi = mid;
        }
        rank += lo;
      }
      if (rank < P.k) out[rank] = e;
    }
  }
}

int lmhead_mma_grid(int ntiles) {
  const int by_tiles = (ntiles + LMM_WARPS - 1) / LMM_WARPS;
  return by_tiles < sm_count() ? by_tiles : sm_count();
}

// Ring depth: as deep as 200 KB of dynamic shared memory allows (2..4).
static size_t lmm_smem(const LmHeadParams& P, int ring) {
  return gm_act_bytes(P.g, P.g.nb) + (lmm_list_bytes(P) + 15) / 16 * 16 +
         size_t(LMM_WARPS) * ring * gm_slot_bytes(P.g);
}

cudaError_t launch_lmhead_mma(LmHeadParams& P, int grid, cudaStream_t stream) {
  if (P.g.ncols < 1 || P.g.ncols > GM_COLS || P.g.split != 1 || P.g.bps != P.g.nb) return cudaErrorInvalidValue;
  int ring = 4;
  while (ring > 2 && lmm_smem(P, ring) > size_t(GEMV_MAX_SMEM)) --ring;
  const size_t smem = lmm_smem(P, ring);
  if (smem > size_t(GEMV_MAX_SMEM)) return cudaErrorInvalidValue;
  P.g.ring = ring;
  static std::atomic<uint64_t> attr_set{0};
  const cudaError_t ea = once_per_current_device(attr_set, [] {
    return cudaFuncSetAttribute(hc_lmhead_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_MAX_SMEM);
  });
  if (ea != cudaSuccess) return ea;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(LMM_WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, hc_lmhead_mma_kernel, P);
}

// Top-k candidates of materialized logits (the tensor-core LM head for wide
// inputs): CTA (chunk, column) walks rows [chunk * chunk_rows, +chunk_rows)
// of one column, each of its 4 warps keeping a running list over 32-row
// steps (topk_insert_warp), then the 4 lists are merged by rank into the
// CTA's k candidates at cand[col * col_stride + chunk * k].
__global__ void __launch_bounds__(GEMV_THREADS) hc_logits_topk_kernel(const float* __restrict__ logits, int rows,
                                                                   int chunk_rows, int k, int32_t id_offset,
                                                                   uint64_t* __restrict__ cand, size_t col_stride) {
  __shared__ uint64_t best[GEMV_WARPS_PER_CTA][TOPK_MAX];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col = blockIdx.y, chunk = blockIdx.x;
  for (int i = threadIdx.x; i < GEMV_WARPS_PER_CTA * TOPK_MAX; i += blockDim.x) (&best[0][0])[i] = 0ull;
  __syncthreads();
  const int lo = chunk * chunk_rows, hi = min(rows, lo + chunk_rows);
  const float* src = logits + size_t(col) * rows;
  for (int base = lo + 32 * warp; base < hi; base += 32 * GEMV_WARPS_PER_CTA) {
    const int row = base + lane;
    const uint64_t key = row < hi ? topk_key(src[row], uint32_t(id_offset + row)) : 0ull;
    topk_insert_warp(best[warp], k, key, lane);
  }
  __syncthreads();
  uint64_t* out = cand + size_t(col) * col_stride + size_t(chunk) * k;
  for (int i = threadIdx.x; i < k; i += blockDim.x) out[i] = 0ull;
  __syncthreads();
  for (int t = threadIdx.x; t < GEMV_WARPS_PER_CTA * k; t += blockDim.x) {
    const int w = t / k, i = t % k;
    const uint64_t e = best[w][i];
    if (e == 0ull) continue;
    int rank = i;
    for (int o = 0; o < GEMV_WARPS_PER_CTA; ++o) {
      if (o == w) continue;
      int a = 0, b = k;  // first index whose key is <= e
      while (a < b) {
        const int mid = (a + b) >> 1;
        if (best[o][mid] > e) a = mid + 1;
        else b = mid;
      }
      rank += a;
    }
    if (rank < k) out[rank] = e;
  }
}

cudaError_t launch_logits_topk(const float* logits, int rows, int cols, int k, int32_t id_offset, uint64_t* cand,
                               size_t col_stride, cudaStream_t stream) {
  const dim3 grid(unsigned((rows + LOGITS_CHUNK_ROWS - 1) / LOGITS_CHUNK_ROWS), unsigned(cols));
  hc_logits_topk_kernel<<<grid, GEMV_THREADS, 0, stream>>>(logits, rows, LOGITS_CHUNK_ROWS, k, id_offset, cand,
                                                        col_stride);
  return cudaGetLastError();
}

// Candidate i of column c lives at c*col_stride + (i / group)*group_stride +
// i % group, so both [col][n] and all-gathered [rank][col][k] layouts merge
// without a transpose.
__device__ __forceinline__ uint64_t cand_at(const uint64_t* c, int i, int group, size_t group_stride) {
  return c[size_t(i / group) * group_stride + (i % group)];
}

// Adds `v` to hist[digit] once per group of lanes that share the digit, so
// concentrated digits (all logits share their exponent bits) do not
// serialize on one shared-memory address.
__device__ __forceinline__ void hist_add(unsigned* hist, unsigned digit, unsigned v) {
  const unsigned act = __activemask();
  const unsigned m = __match_any_sync(act, digit);
  if (int(threadIdx.x & 31) == __ffs(m) - 1) atomicAdd(&hist[digit], v * __popc(m));
}

// Appends x to buf[*n] with one shared atomic per warp.
__device__ __forceinline__ void warp_append(uint64_t* buf, int* n, int cap, uint64_t x) {
  const unsigned act = __activemask();
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(act) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(n, __popc(act));
  base = __shfl_sync(act, base, leader);
  const int pos = base + __popc(act & ((1u << lane) - 1));
  if (pos < cap) buf[pos] = x;
}

constexpr int MERGE_THREADS = 1024;
constexpr int MERGE_BUF = 4096;

// Exact fallback: radix-select the k-th largest key among all n candidates
// (8 passes of 8-bit digits; once the keys still in play fit in shared
// memory they are compacted there), then gather the k keys at or above it
// into sel[].
__device__ void radix_select_topk(const uint64_t* c, int n, int group, size_t group_stride, int k, uint64_t* buf,
                                  uint64_t* sel) {
  __shared__ unsigned hist[256];
  __shared__ uint64_t s_prefix;
  __shared__ int s_remain, s_count, nbuf, nsel;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint64_t prefix = 0, mask = 0;
  int remain = k;
  bool in_buf = false;
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    if (in_buf) {
      for (int i = tid; i < nbuf; i += blockDim.x) {
        const uint64_t x = buf[i];
        if ((x & mask) == prefix) hist_add(hist, unsigned(x >> shift) & 255u, 1u);
      }
    } else {
      for (int i = tid; i < n; i += blockDim.x) {
        const uint64_t x = cand_at(c, i, group, group_stride);
        if ((x & mask) == prefix) hist_add(hist, unsigned(x >> shift) & 255u, 1u);
      }
    }
    __syncthreads();
    if (warp == 0) {
      unsigned local[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        local[j] = hist[8 * lane + j];
        tot += local[j];
      }
      unsigned suf = tot;  // inclusive suffix sum over lanes >= this lane
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const unsigned t = __shfl_down_sync(0xffffffffu, suf, off);
        if (lane + off < 32) suf += t;
      }
      const unsigned above = suf - tot;
      if (above < unsigned(remain) && unsigned(remain) <= above + tot) {
        unsigned acc = above;
        int d = 8 * lane;
        for (int j = 7; j >= 0; --j) {
          if (acc + local[j] >= unsigned(remain)) {
            d = 8 * lane + j;
            break;
          }
          acc += local[j];
        }
        s_prefix = prefix | (uint64_t(d) << shift);
        s_remain = remain - int(acc);
        s_count = int(local[d - 8 * lane]);
      }
    }
    __syncthreads();
    prefix = s_prefix;
    remain = s_remain;
    mask |= uint64_t(0xff) << shift;
    if (!in_buf && shift > 0 && s_count <= MERGE_BUF) {
      // the keys still in play fit in shared memory: compact them there
      if (tid == 0) nbuf = 0;
      __syncthreads();
      for (int i = tid; i < n; i += blockDim.x) {
        const uint64_t x = cand_at(c, i, group, group_stride);
        if ((x & mask) == prefix) warp_append(buf, &nbuf, MERGE_BUF, x);
      }
      in_buf = true;
    }
    __syncthreads();
  }
  if (tid == 0) nsel = 0;
  __syncthreads();
  for (int i = tid; i < n; i += blockDim.x) {
    const uint64_t x = cand_at(c, i, group, group_stride);
    if (x >= prefix) warp_append(sel, &nsel, TOPK_MAX, x);
  }
  __syncthreads();
}

// One CTA per column.  The candidates arrive as `lists` descending lists of
// `group` keys (one per producing CTA or rank).  The k-th largest list head
// h is a lower bound of the answer (k heads are >= h), so only each list's
// prefix of keys >= h can be selected; those survivors (typically about k..3k)
// are copied to shared memory and ranked directly.  If more than MERGE_SURV
// survive (adversarial ties), the exact radix selection runs instead.  Ids and
// values are written in rank order, softcap applied after selection as
// mergeTopCandidates does; the selected keys too when keys_out != nullptr.
constexpr int MERGE_SURV = 1024;

__global__ void __launch_bounds__(MERGE_THREADS) hc_topk_merge_kernel(const uint64_t* __restrict__ cand, int n,
                                                                   size_t col_stride, int group, size_t group_stride,
                                                                   int k, float softcap, int32_t* __restrict__ ids,
                                                                   float* __restrict__ vals,
                                                                   uint64_t* __restrict__ keys_out) {
  __shared__ uint64_t buf[MERGE_BUF];
  __shared__ uint64_t sel[TOPK_MAX];
  __shared__ int s_total, s_warp[MERGE_THREADS / 32];
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
  const uint64_t* c = cand + size_t(blockIdx.x) * col_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int lists = (n + group - 1) / group;
  bool fast = lists <= MERGE_BUF && lists <= MERGE_THREADS;
  uint64_t* heads = buf;  // heads first, survivors later (after a barrier)
  if (fast) {
    for (int g = tid; g < lists; g += blockDim.x) heads[g] = cand_at(c, g * group, group, group_stride);
  }
  __syncthreads();
  // h = k-th largest head (distinct keys; empty lists have head 0)
  __shared__ uint64_t s_h;
  if (fast) {
    if (tid == 0) s_h = 0;
    __syncthreads();
    if (lists <= k) {
      // every key of every list may be needed: survivors = all
    } else {
      for (int g = tid; g < lists; g += blockDim.x) {
        const uint64_t x = heads[g];
        int above = 0;
        for (int o = 0; o < lists; ++o) above += heads[o] > x;
        if (above == k - 1) s_h = x;
      }
    }
  }
  __syncthreads();
  const uint64_t h = s_h;
  // survivors per list: prefix of keys >= h (binary search, lists descending)
  int cnt = 0;
  if (fast && tid < lists) {
    const int base = tid * group;
    const int len = min(group, n - base);
    int lo = 0, hi = len;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (cand_at(c, base + mid, group, group_stride) >= h) lo = mid + 1;
      else hi = mid;
    }
    cnt = lo;
  }
  // block exclusive scan of cnt
  int incl = cnt;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += t;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int v = lane < int(blockDim.x / 32) ? s_warp[lane] : 0;
    int inc = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, inc, off);
      if (lane >= off) inc += t;
    }
    if (lane < int(blockDim.x / 32)) s_warp[lane] = inc - v;
    if (lane == 31) s_total = inc;
  }
  __syncthreads();
  const int total = s_total;
  fast = fast && total <= MERGE_SURV && total >= k;
  if (fast) {
    const int off = s_warp[warp] + incl - cnt;
    for (int i = 0; i < cnt; ++i) buf[off + i] = cand_at(c, tid * group + i, group, group_stride);
    __syncthreads();
    for (int t = tid; t < total; t += blockDim.x) {
      const uint64_t x = buf[t];
      int rank = 0;
      for (int o = 0; o < total; ++o) rank += buf[o] > x;
      if (rank < k) sel[rank] = x;
    }
    __syncthreads();
  } else {
    radix_select_topk(c, n, group, group_stride, k, buf, sel);
    // sel[] holds the k keys unordered: order them
    __syncthreads();
    uint64_t x = 0;
    int rank = 0;
    if (tid < k) {
      x = sel[tid];
      for (int j = 0; j < k; ++j) rank += sel[j] > x;
    }
    __syncthreads();
    if (tid < k) sel[rank] = x;
    __syncthreads();
  }
  if (tid < k) {
    const uint64_t x = sel[tid];
    int32_t id;
    float v;
    topk_decode(x, &id, &v);
    if (softcap > 0.0f) v = float(tanh(double(v) / double(softcap)) * double(softcap));
    ids[size_t(blockIdx.x) * k + tid] = id;
    vals[size_t(blockIdx.x) * k + tid] = v;
    if (keys_out) keys_out[size_t(blockIdx.x) * k + tid] = x;
  }
}

int lmhead_grid(int ntiles) { return persistent_grid(ntiles, sm_count() * GEMV_CTAS_PER_SM); }

template <int NC>
static cudaError_t launch_lm_nc(const LmHeadParams& P, int grid, cudaStream_t stream) {
  static std::atomic<uint64_t> attr_set{0};
  const cudaError_t ea = once_per_current_device(attr_set, [] {
    return cudaFuncSetAttribute(hc_lmhead_topk_kernel<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_MAX_SMEM);
  });
  if (ea != cudaSuccess) return ea;
  const size_t smem = gemv_smem_bytes(P.g, P.g.nb);
  if (smem > size_t(GEMV_MAX_SMEM)) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(GEMV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, hc_lmhead_topk_kernel<NC>, P);
}

cudaError_t launch_lmhead_topk(const LmHeadParams& P, int grid, cudaStream_t stream) {
  if (P.g.ncols <= 1) return launch_lm_nc<1>(P, grid, stream);
  if (P.g.ncols <= 2) return launch_lm_nc<2>(P, grid, stream);
  if (P.g.ncols <= 4) return launch_lm_nc<4>(P, grid, stream);
  return launch_lm_nc<8>(P, grid, stream);
}

cudaError_t launch_topk_merge(const uint64_t* cand, int n, size_t col_stride, int group, size_t group_stride, int cols,
                              int k, float softcap, int32_t* ids, float* vals, uint64_t* keys_out,
                              cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(cols));
  cfg.blockDim = dim3(MERGE_THREADS);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, hc_topk_merge_kernel, cand, n, col_stride, group, group_stride, k, softcap, ids, vals,
                            keys_out);
}

}  // namespace hc
