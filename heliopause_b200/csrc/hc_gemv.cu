// hc_gemv.cu -- Q4_K / Q6_K x Q8_K small-M matmul (M = 1..8 per launch).
//
// Replaces the per-row loop of hp_matmul_quantized_prepared_f32 /
// _multi_f32 (packages/engine/wasm-kernels/src/lib.rs:225-426) and the block
// dots vec_dot_q4_k_q8_k_prepared (lib.rs:2117-2172) and
// vec_dot_q6_k_q8_k_prepared (lib.rs:1924-1968).
//
// Decomposition (B200, HBM-bound):
//   * unit = one 256-element block of one 32-row tile: a contiguous 4,608 B
//     (Q4_K) / 6,720 B (Q6_K) region read as 9 / 13 warp-wide 512-byte loads
//     (lane = row, so no cross-lane reduction inside a block);
//   * item = (tile, K part): the K range of every tile is split into `split`
//     parts so the launch has enough warps (~2,000) to keep HBM busy; a warp
//     streams its item's units through a two-deep register buffer;
//   * split 1  : persistent grid, each warp walks whole tiles;
//     split 2/4: the parts of a tile live in one CTA and are summed in shared
//                memory in part order;
//     split 8-32: a cluster of split/4 CTAs per tile, summed through
//                distributed shared memory in rank order;
//     so every result is deterministic;
//   * programmatic dependent launch: each warp loads its first weight unit
//     before griddepcontrol.wait, the activation slice (written by the
//     previous kernel) is staged into shared memory after it.
//
// Integer block sums are exact (dp4a / dp2a on the same int8 operands as the
// reference); the f32 combine of the per-block terms runs in a different
// order than the reference's 8-lane accumulators, so outputs agree to f32
// rounding.
#include <cooperative_groups.h>
#include <cstdlib>

#include "hc_common.cuh"
#include "hc_bulk.cuh"
#include "hc_decmath.cuh"
#include "hc_gemv_body.cuh"
#include "hc_kernels.cuh"
#include "hc_q8.cuh"

namespace cg = cooperative_groups;

namespace hc {

template <int NC>
struct GemvFlush {
  const GemvParams* p;
  float (*red)[NC][32];
  int warp, lane;
  __device__ __forceinline__ void operator()(int item, const float (&v)[NC]) {
    if (p->split == 1) {
      const int tile = item;
      const GemvSeg& sg = p->seg[seg_of(*p, tile)];
      const int row = (tile - sg.tile_begin) * TILE + lane;
      if (row < sg.rows) {
#pragma unroll
        for (int c = 0; c < NC; ++c)
          if (c < p->ncols) sg.out[size_t(p->col0 + c) * sg.rows + row] = v[c];
      }
    } else {
#pragma unroll
      for (int c = 0; c < NC; ++c) red[warp][c][lane] = v[c];
    }
  }
};

template <int NC>
__device__ __forceinline__ void store_tile(const GemvParams& p, int tile, const float (&v)[NC], int lane) {
  const GemvSeg& sg = p.seg[seg_of(p, tile)];
  const int row = (tile - sg.tile_begin) * TILE + lane;
  if (row < sg.rows) {
#pragma unroll
    for (int c = 0; c < NC; ++c)
      if (c < p.ncols) sg.out[size_t(p.col0 + c) * sg.rows + row] = v[c];
  }
}

// The fused prologue (after the wait): for every column, h = x [+
// rmsnorm(y) * w_post] (f64 sums and products rounded to f32 as
// hc_norm_quant_kernel / layers.ts:824-885), n = rmsnorm(h) * w_pre, and the
// blocks of the CTA's slice [kb0, kb0 + nblk) -- each held whole by one warp
// -- quantized to Q8_K into the shared-memory records.  CTA 0 stores h.
__device__ __forceinline__ void gemv_prologue(const GemvParams& p, uint8_t* act_a, uint8_t* act_b, int kb0, int nblk,
                                              int warp, int lane) {
  __shared__ double scratch[GEMV_WARPS_PER_CTA];
  __shared__ __align__(16) uint8_t stage[GEMV_WARPS_PER_CTA][256];
  constexpr int D = GEMV_PRO_D;
  const bool resid = p.pro.mode == GEMV_PRO_RESID_NORM;
  // Thread (warp w, lane L) owns elements 8L..8L+7 of 256-blocks w and w + 4.
  // Loads are issued as late as their use allows without a dependent round
  // trip (w_pre goes out before the last reduction), which keeps the live
  // registers low next to the main loop's unit buffer.
  const int e0 = warp * 256 + 8 * lane, e1 = (warp + 4) * 256 + 8 * lane;
  for (int c = 0; c < p.ncols; ++c) {
    const size_t col = size_t(p.col0 + c) * D;
    float h[16];
    load8(p.pro.x + col + e0, *reinterpret_cast<float(*)[8]>(&h[0]));
    load8(p.pro.x + col + e1, *reinterpret_cast<float(*)[8]>(&h[8]));
    if (resid) {
      float y[16], wpost[16];
      load8(p.pro.y + col + e0, *reinterpret_cast<float(*)[8]>(&y[0]));
      load8(p.pro.y + col + e1, *reinterpret_cast<float(*)[8]>(&y[8]));
      load8(p.pro.w_post + e0, *reinterpret_cast<float(*)[8]>(&wpost[0]));
      load8(p.pro.w_post + e1, *reinterpret_cast<float(*)[8]>(&wpost[8]));
      double ss = 0.0;
#pragma unroll
      for (int i = 0; i < 16; ++i) ss += double(y[i]) * double(y[i]);
      ss = block_sum_d(ss, scratch, GEMV_WARPS_PER_CTA);
      const double sc = 1.0 / sqrt(ss / double(D) + p.pro.eps);
#pragma unroll
      for (int i = 0; i < 16; ++i) h[i] = h[i] + float((double(y[i]) * sc) * double(wpost[i]));
      if (blockIdx.x == 0) {
        float* xo = p.pro.x_out + col;
        reinterpret_cast<float4*>(xo + e0)[0] = make_float4(h[0], h[1], h[2], h[3]);
        reinterpret_cast<float4*>(xo + e0)[1] = make_float4(h[4], h[5], h[6], h[7]);
        reinterpret_cast<float4*>(xo + e1)[0] = make_float4(h[8], h[9], h[10], h[11]);
        reinterpret_cast<float4*>(xo + e1)[1] = make_float4(h[12], h[13], h[14], h[15]);
      }
    }
    float wpre[16];
    load8(p.pro.w_pre + e0, *reinterpret_cast<float(*)[8]>(&wpre[0]));
    load8(p.pro.w_pre + e1, *reinterpret_cast<float(*)[8]>(&wpre[8]));
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < 16; ++i) ss += double(h[i]) * double(h[i]);
    ss = block_sum_d(ss, scratch, GEMV_WARPS_PER_CTA);
    const double sc = 1.0 / sqrt(ss / double(D) + p.pro.eps);
#pragma unroll
    for (int i = 0; i < 16; ++i) h[i] = float((double(h[i]) * sc) * double(wpre[i]));
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int b = warp + 4 * k;
      if (b >= kb0 && b < kb0 + nblk) {
        const size_t r = size_t(c) * nblk + (b - kb0);
        q8k_block_warp(*reinterpret_cast<const float(*)[8]>(&h[8 * k]), lane, stage[warp], act_a + r * Q8A_REC,
                       act_b + r * Q8B_REC);
      }
    }
  }
}

// Stages the activation slice: bulk copies of the Q8_K records written by the
// previous kernel, or the fused prologue.  Every thread calls it after the
// wait; on return the slice is complete for the whole CTA.
__device__ __forceinline__ void gemv_inputs(const GemvParams& p, uint8_t* act_a, uint8_t* act_b, int kb0, int nblk,
                                            uint64_t* act_bar, int warp, int lane) {
  if (p.pro.mode != GEMV_PRO_NONE) {
    gemv_prologue(p, act_a, act_b, kb0, nblk, warp, lane);
    __syncthreads();
    return;
  }
  stage_activations_bulk(p, act_a, act_b, kb0, nblk, act_bar);
  __syncthreads();
  mbar_wait_parity(act_bar, 0, p.err);
}

// UC: register-buffer chunks per unit (Q6K_CHUNKS, or Q4K_CHUNKS for Q4_K-only
// launches, which then fit GEMV_CTAS_PER_SM_Q4 CTAs per SM).
template <int NC, int UC>
__global__ void __launch_bounds__(GEMV_THREADS, UC == Q4K_CHUNKS ? GEMV_CTAS_PER_SM_Q4 : GEMV_CTAS_PER_SM)
    hc_gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[GEMV_WARPS_PER_CTA][NC][32];
  __shared__ __align__(8) uint64_t act_bar;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.launch_dependents;");
#endif
  const int nitems = p.total_tiles * p.split;
  int item0, istride, kb0 = 0, nblk = p.nb;
  if (p.split == 1) {  // warps walk whole tiles (persistent unless bulk)
    item0 = blockIdx.x * GEMV_WARPS_PER_CTA + warp;
    istride = p.bulk ? nitems : gridDim.x * GEMV_WARPS_PER_CTA;
  } else if (p.split <= GEMV_WARPS_PER_CTA) {  // one item per warp, a tile's parts in one CTA
    item0 = blockIdx.x * GEMV_WARPS_PER_CTA + warp;
    istride = nitems;
  } else {  // one tile per cluster, rank r owns parts [4r, 4r + 4)
    const int csize = p.split / GEMV_WARPS_PER_CTA;
    const int tile = blockIdx.x / csize, rank = blockIdx.x % csize;
    item0 = tile * p.split + rank * GEMV_WARPS_PER_CTA + warp;
    istride = nitems;
    kb0 = rank * GEMV_WARPS_PER_CTA * p.bps;
    nblk = GEMV_WARPS_PER_CTA * p.bps;
  }

  bool need_a, need_b;
  gemv_planes(p, &need_a, &need_b);
  uint8_t* act_a = need_a ? smem : nullptr;
  uint8_t* act_b = need_b ? smem + (need_a ? size_t(p.ncols) * nblk * Q8A_REC : 0) : nullptr;
  const ActSlice act{act_a, act_b, nblk, kb0};
  GemvFlush<NC> flush{&p, red, warp, lane};

  if (p.bulk) {
    // Bulk mode (one item per warp): copy every unit of the CTA into shared
    // memory before waiting for the previous kernel, then compute from there.
    __shared__ __align__(8) uint64_t bar;
    uint8_t* units = smem + (gemv_smem_bytes(p, nblk) + 15) / 16 * 16;  // after the activation slice
    const int ub_max = unit_bytes(UC == Q4K_CHUNKS ? TYPE_Q4_K : TYPE_Q6_K);
    if (threadIdx.x == 0) {
      mbar_init(&bar, 1);
      uint32_t total = 0;
      for (int w = 0; w < GEMV_WARPS_PER_CTA; ++w) {
        const int it = item0 - warp + w;
        if (it >= nitems) break;
        for (int jj = 0; jj < p.bps; ++jj) {
          int t;
          unit_addr(p, it, jj, &t);
          total += uint32_t(unit_bytes(t));
        }
      }
      mbar_expect_tx(&bar, total);
      for (int w = 0; w < GEMV_WARPS_PER_CTA; ++w) {
        const int it = item0 - warp + w;
        if (it >= nitems) break;
        for (int jj = 0; jj < p.bps; ++jj) {
          int t;
          const uint8_t* src = unit_addr(p, it, jj, &t);
          bulk_copy_g2s(units + size_t(w * p.bps + jj) * ub_max, src, uint32_t(unit_bytes(t)), &bar);
        }
      }
    }
#if __CUDA_ARCH__ >= 900
    asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
    gemv_inputs(p, act_a, act_b, kb0, nblk, &act_bar, warp, lane);
    const bool ok = mbar_wait_parity(&bar, 0, p.err);
    if (item0 < nitems) {
      float acc[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) acc[c] = 0.0f;
      if (ok) {
        int t;
        unit_addr(p, item0, 0, &t);
        for (int jj = 0; jj < p.bps; ++jj) {
          UnitRegsN<UC> r;
          load_unit_smem<UC>(r, units + size_t(warp * p.bps + jj) * ub_max, t, lane);
          unit_compute<NC, UC>(r, t, (item0 & (p.split - 1)) * p.bps + jj - kb0, p.ncols, act, acc);
        }
      }
      flush(item0, acc);
    }
  } else {
    UnitRegsN<UC> buf[2];
    int first_type = TYPE_Q4_K;
    __shared__ __align__(8) uint64_t pre_bar[GEMV_WARPS_PER_CTA];
    const int ub_max = unit_bytes(UC == Q4K_CHUNKS ? TYPE_Q4_K : TYPE_Q6_K);
    uint8_t* staged = smem + (gemv_smem_bytes(p, nblk) + 15) / 16 * 16 + size_t(warp) * p.pre * ub_max;
    if (item0 < nitems) {
      load_unit<UC>(buf[0], unit_addr(p, item0, 0, &first_type), first_type, lane);
      if (p.pre > 0 && lane == 0) {
        // units 1..pre of this warp's item into its shared-memory slots
        const uint32_t ub = uint32_t(unit_bytes(first_type));
        mbar_init(&pre_bar[warp], 1);
        mbar_expect_tx(&pre_bar[warp], ub * uint32_t(p.pre));
        for (int jj = 1; jj <= p.pre; ++jj) {
          int t;
          bulk_copy_g2s(staged + size_t(jj - 1) * ub_max, unit_addr(p, item0, jj, &t), ub, &pre_bar[warp]);
        }
      }
      __syncwarp();
    }
#if __CUDA_ARCH__ >= 900
    asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
    gemv_inputs(p, act_a, act_b, kb0, nblk, &act_bar, warp, lane);
    if (p.pre > 0) {
      if (item0 < nitems)
        prefetched_item<NC, UC>(p, act, item0, lane, buf[0], first_type, staged, ub_max, &pre_bar[warp], flush);
    } else {
      stream_items<NC, UC>(p, act, item0, istride, nitems, lane, buf[0], first_type, flush);
    }
  }
  if (p.split == 1) return;

  __syncthreads();
  if (p.split <= GEMV_WARPS_PER_CTA) {
    // warps holding part 0 of a tile sum the tile's parts in part order
    if (item0 < nitems && item0 % p.split == 0) {
      float v[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        v[c] = red[warp][c][lane];
        for (int k = 1; k < p.split; ++k) v[c] += red[warp + k][c][lane];
      }
      store_tile<NC>(p, item0 / p.split, v, lane);
    }
    return;
  }
  // cluster split: every rank stores its CTA partial (warp order) into its
  // slot of rank 0's gather array; after one cluster barrier rank 0 sums the
  // slots in rank order (so only rank 0's own shared memory is read late)
  __shared__ float gather[GEMV_MAX_CLUSTER][NC][32];
  cg::cluster_group cl = cg::this_cluster();
  const int csize = p.split / GEMV_WARPS_PER_CTA, rank = blockIdx.x % csize;
  if (warp == 0) {
    float* dst = cl.map_shared_rank(&gather[0][0][0], 0) + rank * NC * 32;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float v = red[0][c][lane];
#pragma unroll
      for (int w = 1; w < GEMV_WARPS_PER_CTA; ++w) v += red[w][c][lane];
      dst[c * 32 + lane] = v;
    }
  }
  cl.sync();
  if (rank == 0 && warp == 0) {
    float v[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) v[c] = 0.0f;
    for (int r = 0; r < csize; ++r) {
#pragma unroll
      for (int c = 0; c < NC; ++c) v[c] += gather[r][c][lane];
    }
    store_tile<NC>(p, blockIdx.x / csize, v, lane);
  }
}

int sm_count() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

int persistent_grid_w(int items, int cap, int warps_per_cta) {
  const int warps_cap = cap * warps_per_cta;
  const int per = (items + warps_cap - 1) / warps_cap;                   // items per warp
  const int warps = (items + per - 1) / per;                             // warps needed
  return (warps + warps_per_cta - 1) / warps_per_cta;
}

int persistent_grid(int items, int cap) { return persistent_grid_w(items, cap, GEMV_WARPS_PER_CTA); }

static int ctas_per_sm(const GemvParams& p) { return p.q4small ? GEMV_CTAS_PER_SM_Q4 : GEMV_CTAS_PER_SM; }

// Per-SM shared memory a streaming launch may fill with prefetched units:
// GEMV_PRE_SM_SMEM, or HPC_GEMV_PREFETCH_KB (0 turns prefetching off).
static long gemv_pre_sm_smem() {
  static long v = -1;
  if (v < 0) {
    const char* e = getenv("HPC_GEMV_PREFETCH_KB");
    v = e ? atol(e) * 1024 : long(GEMV_PRE_SM_SMEM);
    if (v < 0) v = 0;
  }
  return v;
}

void gemv_plan(GemvParams& p) {
  // Split K as far as the launch still fits in one wave of resident CTAs
  // (ctas_per_sm per SM, one item per warp); parts stay >= 1 block and the
  // cluster form is used up to 8 CTAs (split 32).
  p.q4small = p.ncols <= 2;
  for (int i = 0; i < p.nseg; ++i)
    if (p.seg[i].type != TYPE_Q4_K) p.q4small = 0;
  const int cap_warps = sm_count() * ctas_per_sm(p) * GEMV_WARPS_PER_CTA;
  int s = 1, lg = 0;
  const int smax = p.pro.mode != GEMV_PRO_NONE ? 8 : 32;  // a prologue slice is >= 4 aligned blocks
  while (s < smax && p.nb % (s * 2) == 0 && p.total_tiles * s * 2 <= cap_warps) {
    s *= 2;
    ++lg;
  }
  p.split = s;
  p.split_log2 = lg;
  p.bps = p.nb / s;
  // Launches that fit in one wave stage all their units in shared memory --
  // one wave counting the CTAs that the staged units leave room for.
  const size_t unit_smem = size_t(GEMV_WARPS_PER_CTA) * p.bps * unit_bytes(p.q4small ? TYPE_Q4_K : TYPE_Q6_K);
  const int nblk = p.split > GEMV_WARPS_PER_CTA ? GEMV_WARPS_PER_CTA * p.bps : p.nb;
  const size_t cta_smem = unit_smem + gemv_smem_bytes(p, nblk) + gemv_static_smem(p.ncols);
  const int by_smem = int(size_t(GEMV_SM_SMEM) / cta_smem);
  const int bulk_ctas = sm_count() * (by_smem < ctas_per_sm(p) ? by_smem : ctas_per_sm(p));
  const int grid_items = (p.total_tiles * p.split + GEMV_WARPS_PER_CTA - 1) / GEMV_WARPS_PER_CTA;
  p.bulk = (p.split > 1 || p.total_tiles <= cap_warps) && unit_smem <= size_t(GEMV_BULK_MAX_UNITS_SMEM) &&
           grid_items <= bulk_ctas;
  if (p.split == 1 && p.bulk) {
    // one item per warp in bulk mode: make the grid non-persistent
    p.bulk = p.total_tiles <= cap_warps;
  }
  // Streaming launches of one or two columns with one item per warp
  // prefetch units 1..pre of each item into shared memory before waiting for
  // the previous kernel, as many as fit in GEMV_PRE_SM_SMEM shared by the
  // CTAs that share an SM.  (Wider launches measured slower with it: the
  // larger activation slices leave room for one unit at most.)
  p.pre = 0;
  if (!p.bulk && p.split > 1 && p.bps > 1 && p.ncols <= 2) {
    const int ub = unit_bytes(p.q4small ? TYPE_Q4_K : TYPE_Q6_K);
    const int per_sm = (grid_items + sm_count() - 1) / sm_count();
    const long budget = long(gemv_pre_sm_smem() / per_sm) - long(gemv_smem_bytes(p, nblk)) -
                        long(gemv_static_smem(p.ncols)) - 16;
    const int pre = budget > 0 ? int(budget / (long(GEMV_WARPS_PER_CTA) * ub)) : 0;
    p.pre = pre < p.bps - 1 ? pre : p.bps - 1;
  }
  p.err = device_status_word();
}

int gemv_grid(const GemvParams& p) {
  const int items = p.total_tiles * p.split;
  if (p.split == 1 && !p.bulk) return persistent_grid(items, sm_count() * ctas_per_sm(p));
  return (items + GEMV_WARPS_PER_CTA - 1) / GEMV_WARPS_PER_CTA;
}

template <int NC, int UC>
static cudaError_t launch_nc(const GemvParams& p, cudaStream_t stream) {
  const int nblk = p.split > GEMV_WARPS_PER_CTA ? GEMV_WARPS_PER_CTA * p.bps : p.nb;
  size_t smem = (gemv_smem_bytes(p, nblk) + 15) / 16 * 16;
  if (p.bulk) smem += size_t(GEMV_WARPS_PER_CTA) * p.bps * unit_bytes(UC == Q4K_CHUNKS ? TYPE_Q4_K : TYPE_Q6_K);
  else smem += size_t(GEMV_WARPS_PER_CTA) * p.pre * unit_bytes(UC == Q4K_CHUNKS ? TYPE_Q4_K : TYPE_Q6_K);
  if (smem > size_t(GEMV_MAX_SMEM)) return cudaErrorInvalidValue;
  static std::atomic<uint64_t> attr_set{0};
  const cudaError_t ea = once_per_current_device(attr_set, [] {
    return cudaFuncSetAttribute(hc_gemv_kernel<NC, UC>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_MAX_SMEM);
  });
  if (ea != cudaSuccess) return ea;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(gemv_grid(p)));
  cfg.blockDim = dim3(GEMV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  ++na;
  if (p.split > GEMV_WARPS_PER_CTA) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = unsigned(p.split / GEMV_WARPS_PER_CTA);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, hc_gemv_kernel<NC, UC>, p);
}

cudaError_t launch_gemv(const GemvParams& p, cudaStream_t stream) {
  if (p.q4small) {
    if (p.ncols <= 1) return launch_nc<1, Q4K_CHUNKS>(p, stream);
    return launch_nc<2, Q4K_CHUNKS>(p, stream);
  }
  if (p.ncols <= 1) return launch_nc<1, Q6K_CHUNKS>(p, stream);
  if (p.ncols <= 2) return launch_nc<2, Q6K_CHUNKS>(p, stream);
  if (p.ncols <= 4) return launch_nc<4, Q6K_CHUNKS>(p, stream);
  return launch_nc<8, Q6K_CHUNKS>(p, stream);
}

}  // namespace hc
