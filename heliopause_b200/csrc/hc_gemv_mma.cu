// hc_gemv_mma.cu -- Q4_K / Q6_K x Q8_K GEMV for 3..8 columns on the tensor
// cores (the MTP verify width M = 5, batched decode up to 8).
//
// Replaces the same reference loops as the dp4a GEMV (hc_gemv.cu:
// hp_matmul_quantized_prepared_f32 / _multi_f32, lib.rs:225-426, with the
// block dots of lib.rs:2117-2172 / 1924-1968).  The dp4a GEMV issues one
// dp4a per 4 weights per column, so its cost grows with the column count and
// it becomes compute-bound above two columns.  Here one m16n8 s8 mma covers
// 16 rows x 8 columns, so 3..8 columns cost the same as 8: the block
// products of hc_mma.cuh with one 8-column group.
//
// Decomposition (HBM-bound, as hc_gemv.cu):
//   * unit = one 256-block of one 32-row tile (4,608 / 6,720 B contiguous);
//     item = (tile, K part); a warp streams its items' units through its own
//     ring of `p.ring` shared-memory slots, one cp.async.bulk per unit
//     completing on the slot's mbarrier, refilled as soon as the warp has
//     consumed a slot;
//   * the first ring fill is issued before griddepcontrol.wait (the weights
//     do not depend on the previous kernel); the CTA's activation slice (8
//     columns, columns >= ncols repeat the last one) arrives by bulk copy
//     after it;
//   * CTAs of W = 8 warps (two per SM) share one activation slice, so an SM
//     keeps 16 warps' unit streams in flight: the per-unit work is a chain of
//     shared-memory loads, unpacks, mma and integer scaling, and 8 warps per
//     SM left the schedulers mostly idle (ncu: issue active 35%);
//   * split 1: persistent warps walk whole tiles; split 2..W: a tile's parts
//     in one CTA, summed in shared memory in part order; above W: a cluster
//     of split / W CTAs per tile, summed through distributed shared memory in
//     rank order; so every result is deterministic.
// Every wait is bounded (hc_bulk.cuh): on a timeout the warp stops computing,
// waits (bounded) for its copies in flight and the status word says so.
#include <cooperative_groups.h>
#include <cstdlib>

#include "hc_bulk.cuh"
#include "hc_common.cuh"
#include "hc_gemv_body.cuh"
#include "hc_kernels.cuh"
#include "hc_mma.cuh"
#include "hc_mma_stream.cuh"

namespace cg = cooperative_groups;

namespace hc {

constexpr int GM_MAX_RING = 4;
constexpr int GM_MIN_RING = 2;
constexpr int GM_MAX_CLUSTER = 8;
// Warps per CTA (W) and the resident CTAs its launch bounds ask for: 8 x 2
// by default (HPC_GEMV_MMA_WARPS=4 selects 4 x 3).
template <int W>
struct GmShape {
  static constexpr int THREADS = 32 * W;
  static constexpr int CTAS = W == 8 ? 2 : 3;
  static constexpr size_t STATIC_SMEM = size_t(W + GM_MAX_CLUSTER) * GM_COLS * 32 * 4 + (W * GM_MAX_RING + 1) * 8 + 64;
};

template <int GM_WARPS>
__global__ void __launch_bounds__(GmShape<GM_WARPS>::THREADS, GmShape<GM_WARPS>::CTAS)
    hc_gemv_mma_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[GM_WARPS][GM_COLS][32];
  __shared__ __align__(8) uint64_t bars[GM_WARPS][GM_MAX_RING];
  __shared__ __align__(8) uint64_t act_bar;
  const int lane = int(threadIdx.x & 31), warp = int(threadIdx.x >> 5), g = lane >> 2, t = lane & 3;
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.launch_dependents;");
#endif
  const int nitems = p.total_tiles * p.split;
  int item0, istride, kb0 = 0, nblk = p.nb;
  if (p.split == 1) {
    item0 = int(blockIdx.x) * GM_WARPS + warp;
    istride = int(gridDim.x) * GM_WARPS;
  } else if (p.split <= GM_WARPS) {
    item0 = int(blockIdx.x) * GM_WARPS + warp;
    istride = nitems;
  } else {
    const int csize = p.split / GM_WARPS;
    const int tile = int(blockIdx.x) / csize, rank = int(blockIdx.x) % csize;
    item0 = tile * p.split + rank * GM_WARPS + warp;
    istride = nitems;
    kb0 = rank * GM_WARPS * p.bps;
    nblk = GM_WARPS * p.bps;
  }
  bool need_a, need_b;
  gemv_planes(p, &need_a, &need_b);
  const int cs_a = gm_col_stride(nblk, Q8A_REC), cs_b = gm_col_stride(nblk, Q8B_REC);
  uint8_t* act_a = need_a ? smem : nullptr;
  uint8_t* act_b = need_b ? smem + (need_a ? size_t(GM_COLS) * cs_a : 0) : nullptr;
  const int slot = gm_slot_bytes(p);
  MmaStream ms(p, item0, istride, nitems, smem + gm_act_bytes(p, nblk) + size_t(warp) * p.ring * slot, slot,
               bars[warp], lane);
  ms.prime();
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
  stage_act_slice8(p, act_a, act_b, cs_a, cs_b, kb0, nblk, &act_bar);
  __syncthreads();
  bool ok = mbar_wait_parity(&act_bar, 0, p.err);
  auto flush = [&](int item, const float (&acc)[2][1][4]) {
    const int tile = item >> p.split_log2;
#pragma unroll
    for (int mg = 0; mg < 2; ++mg)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int row = 16 * mg + g + 8 * (r >> 1), col = 2 * t + (r & 1);
        if (p.split == 1) {
          const GemvSeg& sg = p.seg[seg_of(p, tile)];
          const int grow = (tile - sg.tile_begin) * TILE + row;
          if (grow < sg.rows && col < p.ncols) sg.out[size_t(p.col0 + col) * sg.rows + grow] = acc[mg][0][r];
        } else {
          red[warp][col][row] = acc[mg][0][r];
        }
      }
  };
  ok = ms.run(act_a, act_b, cs_a, cs_b, kb0, ok, g, t, flush);
  if (!ok) {
    if (p.split > 1) {
#pragma unroll
      for (int c = 0; c < GM_COLS; ++c) red[warp][c][lane] = 0.0f;
    }
  }
  if (p.split == 1) return;

  __syncthreads();
  if (p.split <= GM_WARPS) {
    // warps holding part 0 of a tile sum the tile's parts in part order (lane = row)
    if (item0 < nitems && item0 % p.split == 0) {
      float v[GM_COLS];
#pragma unroll
      for (int c = 0; c < GM_COLS; ++c) {
        v[c] = red[warp][c][lane];
        for (int k = 1; k < p.split; ++k) v[c] += red[warp + k][c][lane];
      }
      const int tile = item0 / p.split;
      const GemvSeg& sg = p.seg[seg_of(p, tile)];
      const int row = (tile - sg.tile_begin) * TILE + lane;
      if (row < sg.rows) {
#pragma unroll
        for (int c = 0; c < GM_COLS; ++c)
          if (c < p.ncols) sg.out[size_t(p.col0 + c) * sg.rows + row] = v[c];
      }
    }
    return;
  }
  // cluster split: each rank pushes its CTA partial (warp order) into its slot
  // of rank 0's gather array; after one cluster barrier rank 0 sums the slots
  // in rank order
  __shared__ float gather[GM_MAX_CLUSTER][GM_COLS][32];
  cg::cluster_group cl = cg::this_cluster();
  const int csize = p.split / GM_WARPS, rank = int(blockIdx.x) % csize;
  if (warp == 0) {
    float* dst = cl.map_shared_rank(&gather[0][0][0], 0) + rank * GM_COLS * 32;
#pragma unroll
    for (int c = 0; c < GM_COLS; ++c) {
      float v = red[0][c][lane];
#pragma unroll
      for (int w = 1; w < GM_WARPS; ++w) v += red[w][c][lane];
      dst[c * 32 + lane] = v;
    }
  }
  cl.sync();
  if (rank == 0 && warp == 0) {
    float v[GM_COLS];
#pragma unroll
    for (int c = 0; c < GM_COLS; ++c) v[c] = 0.0f;
    for (int r = 0; r < csize; ++r) {
#pragma unroll
      for (int c = 0; c < GM_COLS; ++c) v[c] += gather[r][c][lane];
    }
    const int tile = int(blockIdx.x) / csize;
    const GemvSeg& sg = p.seg[seg_of(p, tile)];
    const int row = (tile - sg.tile_begin) * TILE + lane;
    if (row < sg.rows) {
#pragma unroll
      for (int c = 0; c < GM_COLS; ++c)
        if (c < p.ncols) sg.out[size_t(p.col0 + c) * sg.rows + row] = v[c];
    }
  }
}

// CTAs of `smem` dynamic bytes that fit on one SM.
template <int W>
static int gm_ctas_by_smem(size_t smem) {
  const int n = int(size_t(GEMV_SM_SMEM) / (smem + GmShape<W>::STATIC_SMEM + 1024));
  return n < GmShape<W>::CTAS ? n : GmShape<W>::CTAS;
}

// Split, ring depth and grid of a launch.  The split (parts >= 1 block; a
// cluster of split / W CTAs per tile above W, up to GM_MAX_CLUSTER) is the
// largest whose items all fit in one wave of resident warps at the
// shallowest ring; when none does, the smallest whose shared memory fits (a
// persistent grid at split 1).  The ring is then made as deep as shared
// memory allows (up to GM_MAX_RING) without lowering the resident CTAs per SM.
template <int W>
static void gemv_mma_plan(GemvParams& p, int* grid, size_t* smem) {
  p.bulk = 0;
  p.pre = 0;
  p.q4small = 0;
  const int slot = gm_slot_bytes(p);
  auto smem_for = [&](int split, int ring) {
    const int bps = p.nb / split;
    const int nblk = split > W ? W * bps : p.nb;
    return gm_act_bytes(p, nblk) + size_t(W) * ring * slot;
  };
  int best = 0, fits = 0;
  for (int s = 1; s <= W * GM_MAX_CLUSTER && p.nb % s == 0; s *= 2) {
    const size_t sm = smem_for(s, GM_MIN_RING);
    if (sm > size_t(GEMV_MAX_SMEM)) continue;
    if (!fits) fits = s;
    const int per_sm = gm_ctas_by_smem<W>(sm);
    if (per_sm >= 1 && size_t(p.total_tiles) * s <= size_t(sm_count()) * per_sm * W) best = s;
  }
  const int s = best ? best : fits;
  int lg = 0;
  while ((1 << lg) < s) ++lg;
  p.split = s;
  p.split_log2 = lg;
  p.bps = s ? p.nb / s : 0;
  const int floor_ctas = s ? gm_ctas_by_smem<W>(smem_for(s, GM_MIN_RING)) : 0;
  int ring = GM_MAX_RING;
  while (ring > GM_MIN_RING &&
         (smem_for(s, ring) > size_t(GEMV_MAX_SMEM) || gm_ctas_by_smem<W>(smem_for(s, ring)) < floor_ctas))
    --ring;
  p.ring = ring;
  *smem = s ? smem_for(s, ring) : ~size_t(0);
  const int items = p.total_tiles * s;
  if (s == 1) {
    const int per_sm = gm_ctas_by_smem<W>(*smem);
    *grid = persistent_grid_w(items, sm_count() * (per_sm > 0 ? per_sm : 1), W);
  } else {
    *grid = (items + W - 1) / W;
  }
  p.err = device_status_word();
}

template <int W>
static cudaError_t launch_gemv_mma_w(GemvParams& p, cudaStream_t stream) {
  int grid;
  size_t smem;
  gemv_mma_plan<W>(p, &grid, &smem);
  if (p.split == 0 || smem > size_t(GEMV_MAX_SMEM)) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_set{0};
  const cudaError_t ea = once_per_current_device(attr_set, [] {
    return cudaFuncSetAttribute(hc_gemv_mma_kernel<W>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_MAX_SMEM);
  });
  if (ea != cudaSuccess) return ea;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(GmShape<W>::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  ++na;
  if (p.split > W) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = unsigned(p.split / W);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, hc_gemv_mma_kernel<W>, p);
}

static int gemv_mma_warps() {
  static int v = 0;
  if (!v) {
    const char* e = getenv("HPC_GEMV_MMA_WARPS");
    v = e && atoi(e) == 4 ? 4 : 8;
  }
  return v;
}

cudaError_t launch_gemv_mma(GemvParams& p, cudaStream_t stream) {
  if (p.ncols < 1 || p.ncols > GM_COLS || p.pro.mode != GEMV_PRO_NONE) return cudaErrorInvalidValue;
  return gemv_mma_warps() == 4 ? launch_gemv_mma_w<4>(p, stream) : launch_gemv_mma_w<8>(p, stream);
}

}  // namespace hc
