// hc_gemvx.cu -- Q4_K / Q6_K x Q8_K small-M matmul (1..8 columns per
// launch) whose every row dot equals vec_dot_q4_k_q8_k_prepared /
// vec_dot_q6_k_q8_k_prepared (lib.rs:2117-2172 / 1924-1968) bit for bit:
// the reference's eight f32 lane accumulators advanced block by block in
// block order (hc_exact.cuh).
//
// Decomposition (B200, HBM-bound streaming):
//   * unit = one 256-element block of one 32-row tile (4,608 / 6,720 B
//     contiguous in the row-tile layout), lane = row;
//   * a CTA of 8 warps owns one tile at a time and one contiguous part of
//     its K range (a cluster of C CTAs splits long rows: rank r holds blocks
//     [r*nbc, (r+1)*nbc)); warp w takes the CTA's blocks w, w+8, ...;
//   * each warp streams its units through its own ring of R shared-memory
//     slots (one cp.async.bulk per unit, completion on the slot's mbarrier,
//     refilled as soon as the slot is consumed), primed before
//     griddepcontrol.wait since the weights do not depend on the previous
//     kernel; clusters loop over tiles (persistent grid);
//   * per block and column a warp turns the exact integer lane sums into
//     the reference's nine f32 products (d*aux32[l], dmin*sumi) and parks
//     them in shared memory; after a barrier (cluster barrier when C > 1)
//     one warp per column of rank 0 walks the row's blocks in order,
//     reading other ranks' products through distributed shared memory, and
//     adds them into the nine accumulators exactly as the reference does.
//     The products are double-buffered by tile parity, so the other warps
//     stream the next tile while that chain runs.
// Activations are read as plane-A/B Q8_K records straight from global
// memory (every lane reads the same record words; they stay in L1/L2).
#include <cooperative_groups.h>

#include "hc_bulk.cuh"
#include "hc_common.cuh"
#include "hc_decmath.cuh"
#include "hc_exact.cuh"
#include "hc_gemv_body.cuh"
#include "hc_kernels.cuh"

namespace cg = cooperative_groups;

namespace hc {

namespace {

constexpr int GX_WARPS = 8;
constexpr int GX_THREADS = 32 * GX_WARPS;
constexpr int GX_MAX_R = 4;
constexpr int GX_PROD = 9 * 32;  // floats of one (block, column): 9 products x 32 rows

__device__ __forceinline__ int gx_seg_of(const GemvxParams& p, int tile) {
  int si = 0;
#pragma unroll
  for (int i = 1; i < GEMV_MAXSEG; ++i)
    if (i < p.nseg && tile >= p.seg[i].tile_begin) si = i;
  return si;
}

__host__ __device__ inline size_t gx_prod_floats(int nbc, int nc) { return size_t(nbc) * nc * GX_PROD; }

// Dynamic shared memory, in order: the warps' ring slots [8][R][slot]; the
// products, double-buffered by tile parity [2][nbc][ncols][9][32]; the
// finished accumulators [2][ncols][9][32]; the CTA's activation records,
// plane A [ncols][nbc][288] then plane B [ncols][nbc][304] (the planes the
// launch's weight types use).
__host__ __device__ inline size_t gx_fin_floats(int nc) { return size_t(nc) * GX_PROD; }
__host__ __device__ inline size_t gx_act_bytes(const GemvxParams& p) {
  return size_t(p.ncols) * p.nbc * (((p.planes & 1) ? Q8A_REC : 0) + ((p.planes & 2) ? Q8B_REC : 0));
}
__host__ __device__ inline size_t gx_smem_bytes(const GemvxParams& p) {
  return size_t(GX_WARPS) * p.R * p.slot + 2 * (gx_prod_floats(p.nbc, p.ncols) + gx_fin_floats(p.ncols)) * sizeof(float) +
         gx_act_bytes(p);
}

template <int NC>
__global__ void __launch_bounds__(GX_THREADS, 1) hc_gemvx_kernel(const __grid_constant__ GemvxParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[GX_WARPS * GX_MAX_R];
  const int lane = int(threadIdx.x) & 31, warp = int(threadIdx.x) >> 5;
  pdl_trigger();
  const int C = p.C;
  const int rank = int(blockIdx.x) % C, cid = int(blockIdx.x) / C, ncl = int(gridDim.x) / C;
  const int ntl = cid < p.total_tiles ? (p.total_tiles - 1 - cid) / ncl + 1 : 0;  // tiles of this cluster
  const int bpw = warp < p.nbc ? (p.nbc - 1 - warp) / GX_WARPS + 1 : 0;          // this warp's blocks per tile
  const int n = ntl * bpw;                                                        // this warp's units
  const int R = p.R;
  uint8_t* ring = smem + size_t(warp) * R * p.slot;
  float* prod = reinterpret_cast<float*>(smem + size_t(GX_WARPS) * R * p.slot);  // [2][nbc][ncols][9][32]
  const size_t pstride = gx_prod_floats(p.nbc, p.ncols), fstride = gx_fin_floats(p.ncols);
  float* fin = prod + 2 * pstride;                                                // [2][ncols][9][32]
  uint8_t* act_a = reinterpret_cast<uint8_t*>(fin + 2 * fstride);                 // [ncols][nbc][288]
  uint8_t* act_b = act_a + ((p.planes & 1) ? size_t(p.ncols) * p.nbc * Q8A_REC : 0);  // [ncols][nbc][304]
  __shared__ __align__(8) uint64_t act_bar;
  uint64_t* wb = bars + warp * R;

  // unit u of this warp: tile (u / bpw) of the cluster's list, local block warp + 8 * (u % bpw)
  auto issue = [&](int u) {
    const int tile = cid + (u / bpw) * ncl;
    const int b = rank * p.nbc + warp + GX_WARPS * (u % bpw);
    const GemvSeg& sg = p.seg[gx_seg_of(p, tile)];
    const uint32_t ub = uint32_t(unit_bytes(sg.type));
    uint64_t* bar = wb + (u % R);
    mbar_expect_tx(bar, ub);
    bulk_copy_g2s(ring + size_t(u % R) * p.slot, sg.w + (size_t(tile - sg.tile_begin) * p.nb + b) * ub, ub, bar);
  };
  const int primed = n < R ? n : R;
  if (lane == 0) {
    for (int s = 0; s < R; ++s) mbar_init(wb + s, 1);
    for (int u = 0; u < primed; ++u) issue(u);
  }
  __syncwarp();
  pdl_wait();  // the activation records are written by the previous kernel
  // this CTA's activation records (blocks [rank * nbc, (rank + 1) * nbc) of
  // every column), one bulk copy per column and plane
  if (threadIdx.x == 0) {
    mbar_init(&act_bar, 1);
    mbar_expect_tx(&act_bar, uint32_t(gx_act_bytes(p)));
    for (int c = 0; c < p.ncols; ++c) {
      const size_t rec0 = size_t(p.col0 + c) * p.nb + size_t(rank) * p.nbc;
      if (p.planes & 1)
        bulk_copy_g2s(act_a + size_t(c) * p.nbc * Q8A_REC, p.q.a + rec0 * Q8A_REC, uint32_t(p.nbc * Q8A_REC), &act_bar);
      if (p.planes & 2)
        bulk_copy_g2s(act_b + size_t(c) * p.nbc * Q8B_REC, p.q.b + rec0 * Q8B_REC, uint32_t(p.nbc * Q8B_REC), &act_bar);
    }
  }
  __syncthreads();
  bool ok = mbar_wait_parity(&act_bar, 0, p.err);
  int issued = primed;
  for (int i = 0; i < ntl; ++i) {
    const int tile = cid + i * ncl;
    const GemvSeg& sg = p.seg[gx_seg_of(p, tile)];
    const bool q4 = sg.type == TYPE_Q4_K;
    float* pbuf = prod + size_t(i & 1) * pstride;
    for (int k = 0; k < bpw; ++k) {
      const int u = i * bpw + k;
      if (ok && !mbar_wait_parity_sleep(wb + (u % R), uint32_t(u / R) & 1u, p.err)) ok = false;
      const int jb = warp + GX_WARPS * k;  // block inside this CTA's part
      if (ok) {
        const uint8_t* unit = ring + size_t(u % R) * p.slot;
        const SmemSrc src{reinterpret_cast<const uint4*>(unit) + lane,
                          reinterpret_cast<const uint16_t*>(unit + Q6K_DPLANE_OFFSET) + lane};
        float* pb = pbuf + size_t(jb) * p.ncols * GX_PROD + lane;
        if (q4) {
          const Q4KHeader hd = q4k_header(src.chunk(0));
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            if (c < p.ncols) {
              const uint8_t* rec = act_a + (size_t(c) * p.nbc + jb) * Q8A_REC;
              BlockInts bi;
              q4k_lanes(src, hd, rec, bi);
              const float d8 = *reinterpret_cast<const float*>(rec + Q8A_D);
              const float d = __fmul_rn(hd.d, d8), dm = __fmul_rn(hd.dmin, d8);
              float* o = pb + c * GX_PROD;
#pragma unroll
              for (int l = 0; l < 8; ++l) o[l * 32] = __fmul_rn(d, float(bi.aux[l]));
              o[8 * 32] = __fmul_rn(dm, float(bi.msum));
            }
          }
        } else {
          const float dw = f16_bits_to_f32(src.dbits());
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            if (c < p.ncols) {
              const uint8_t* rec = act_b + (size_t(c) * p.nbc + jb) * Q8B_REC;
              BlockInts bi;
              q6k_lanes(src, rec, bi);
              const float d = __fmul_rn(dw, *reinterpret_cast<const float*>(rec + Q8B_D));
              float* o = pb + c * GX_PROD;
#pragma unroll
              for (int l = 0; l < 8; ++l) o[l * 32] = __fmul_rn(d, float(bi.aux[l]));
              o[8 * 32] = 0.0f;
            }
          }
        }
      }
      __syncwarp();  // every lane has read the slot: refill it
      if (u + R < n) {
        if (ok && lane == 0) issue(u + R);
        if (ok) ++issued;
      }
    }
    // every part's products of this tile are in place
    if (C > 1) cg::this_cluster().sync();
    else __syncthreads();
    if (rank == 0) {
      // rank 0 walks the row's blocks in order: warp w advances lane
      // accumulator w of every column (warp 0 also sumf), reading the other
      // ranks' products through distributed shared memory
      float* f = fin + size_t(i & 1) * fstride;
      const float* pb = prod + size_t(i & 1) * pstride;
      if (ok) {
        for (int c = 0; c < p.ncols; ++c) {
          for (int kk = warp; kk < 9; kk += GX_WARPS) {
            float acc = 0.0f;
            const float* base = pb + (size_t(c) * 9 + kk) * 32 + lane;
#pragma unroll 8
            for (int b = 0; b < p.nb; ++b) {
              const int r = b / p.nbc, jb = b - r * p.nbc;
              const float* src = base + size_t(jb) * p.ncols * GX_PROD;
              if (C > 1 && r != 0) src = cg::this_cluster().map_shared_rank(src, r);
              acc = kk < 8 ? __fadd_rn(acc, *src) : __fsub_rn(acc, *src);
            }
            f[(c * 9 + kk) * 32 + lane] = acc;
          }
        }
      }
      __syncthreads();
      if (ok && warp < NC && warp < p.ncols) {  // one warp per column: sumf + the lane total
        const float* fc = f + warp * GX_PROD + lane;
        float t = 0.0f;
#pragma unroll
        for (int l = 0; l < 8; ++l) t = __fadd_rn(t, fc[l * 32]);
        const float v = q4 ? __fadd_rn(fc[8 * 32], t) : t;
        const int row = (tile - sg.tile_begin) * TILE + lane;
        if (row < sg.rows) sg.out[size_t(p.col0 + warp) * sg.rows + row] = v;
      }
    }
  }
  // rank 0 reads the other ranks' products until its last chain is done
  if (C > 1) cg::this_cluster().sync();
  if (!ok)
    for (int u = n < issued ? n : issued, v = 0; v < u; ++v) mbar_wait_parity(wb + (v % R), uint32_t(v / R) & 1u, nullptr);
}

}  // namespace

int gemvx_plan(GemvxParams& p, int sms) {
  // ring slot: the largest unit among the launch's weights
  p.slot = 0;
  p.planes = 0;
  for (int i = 0; i < p.nseg; ++i) {
    p.slot = max(p.slot, unit_bytes(p.seg[i].type));
    p.planes |= p.seg[i].type == TYPE_Q4_K ? 1 : 2;
  }
  // split long rows over a cluster until the launch covers every SM once
  // (a CTA keeps at least 8 blocks, one per warp), and further while a CTA's
  // products would not fit its shared memory
  p.C = 1;
  auto can_split = [&] { return p.C < 8 && p.nb % (2 * p.C * GX_WARPS) == 0; };
  while (can_split() && p.total_tiles * p.C < sms) p.C *= 2;
  for (;;) {
    p.nbc = p.nb / p.C;
    p.R = 1;
    if (gx_smem_bytes(p) <= size_t(GEMV_MAX_SMEM) || !can_split()) break;
    p.C *= 2;
  }
  // Ring depth R and CTAs per SM: the least work on the busiest SM first
  // (ceil(tiles / clusters) tiles per cluster, times the CTAs that share an
  // SM's bandwidth), then the most unit bytes in flight per SM.
  int best_rounds = 1 << 30, best_ctas = 0, best_r = 0;
  long best_inflight = -1;
  for (int ctas = 2; ctas >= 1; --ctas) {
    for (int r = 1; r <= GX_MAX_R; ++r) {
      p.R = r;
      const size_t limit = ctas == 2 ? size_t(GEMV_SM_SMEM) / 2 - 2048 : size_t(GEMV_MAX_SMEM);
      if (gx_smem_bytes(p) > limit) break;
      const int cl = min(p.total_tiles, max(1, sms * ctas / p.C));
      const int rounds = (p.total_tiles + cl - 1) / cl * ctas;
      const long inflight = long(ctas) * GX_WARPS * r * p.slot;
      if (rounds < best_rounds || (rounds == best_rounds && inflight > best_inflight)) {
        best_rounds = rounds;
        best_inflight = inflight;
        best_ctas = ctas;
        best_r = r;
      }
    }
  }
  if (best_ctas == 0) return -1;
  p.R = best_r;
  const int clusters = min(p.total_tiles, max(1, sms * best_ctas / p.C));
  p.err = device_status_word();
  return clusters * p.C;
}

template <int NC>
static cudaError_t launch_x(const GemvxParams& p, int grid, cudaStream_t st) {
  const size_t smem = gx_smem_bytes(p);
  static std::atomic<uint64_t> attr_set{0};
  const cudaError_t ea = once_per_current_device(attr_set, [] {
    return cudaFuncSetAttribute(hc_gemvx_kernel<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_MAX_SMEM);
  });
  if (ea != cudaSuccess) return ea;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(GX_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  ++na;
  if (p.C > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = unsigned(p.C);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, hc_gemvx_kernel<NC>, p);
}

cudaError_t launch_gemvx(GemvxParams& p, cudaStream_t st) {
  if (p.ncols < 1 || p.ncols > GEMVX_MAX_COLS) return cudaErrorInvalidValue;
  const int grid = gemvx_plan(p, sm_count());
  if (grid <= 0) return cudaErrorInvalidValue;
  if (p.ncols <= 1) return launch_x<1>(p, grid, st);
  if (p.ncols <= 2) return launch_x<2>(p, grid, st);
  if (p.ncols <= 4) return launch_x<4>(p, grid, st);
  return launch_x<8>(p, grid, st);
}

}  // namespace hc
