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

#include <cstdlib>

#include "hc_bulk.cuh"
#include "hc_common.cuh"
#include "hc_decmath.cuh"
#include "hc_exact.cuh"
#include "hc_gemv_body.cuh"
#include "hc_kernels.cuh"
#include "hc_mma.cuh"
#include "hc_q8.cuh"

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

// The prologue (after the wait): warp w holds 256-block w of the width-2048
// input (lane L: elements 256w + 8L .. +7), as hc_norm_quant_kernel does, and
// every step rounds as there: for each column, RESID_NORM h = x +
// f32((y * s_y) * w_post) (CTA 0 stores h to x_out), NORM / RESID_NORM
// n = f32((h * s_h) * w_pre) with s = 1 / sqrt(sum of squares / D + eps) in
// f64, QUANT n = x; then the blocks of this CTA's part are quantized to Q8_K
// straight into its shared-memory records.
__device__ __forceinline__ void gx_prologue(const GemvxParams& p, uint8_t* act_a, uint8_t* act_b, int rank, int warp,
                                            int lane) {
  __shared__ double scratch[GX_WARPS];
  constexpr int D = GEMV_PRO_D;
  const GemvPrologue& pro = p.pro;
  const int e0 = warp * 256 + 8 * lane;
  float wq[8], wp[8];
  if (pro.mode != GEMV_PRO_QUANT) load8(pro.w_pre + e0, wq);
  if (pro.mode == GEMV_PRO_RESID_NORM) load8(pro.w_post + e0, wp);
  for (int c = 0; c < p.ncols; ++c) {
    const size_t col = size_t(p.col0 + c) * D;
    float h[8];
    load8(pro.x + col + e0, h);
    if (pro.mode == GEMV_PRO_RESID_NORM) {
      float y[8];
      load8(pro.y + col + e0, y);
      double ss = 0.0;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += double(y[i]) * double(y[i]);
      ss = block_sum_d(ss, scratch, GX_WARPS);
      const double sc = 1.0 / sqrt(ss / double(D) + pro.eps);
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = h[i] + float((double(y[i]) * sc) * double(wp[i]));
      if (blockIdx.x == 0) {
        float4* xo = reinterpret_cast<float4*>(pro.x_out + col + e0);
        xo[0] = make_float4(h[0], h[1], h[2], h[3]);
        xo[1] = make_float4(h[4], h[5], h[6], h[7]);
      }
    }
    if (pro.mode != GEMV_PRO_QUANT) {
      double ss = 0.0;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += double(h[i]) * double(h[i]);
      ss = block_sum_d(ss, scratch, GX_WARPS);
      const double sc = 1.0 / sqrt(ss / double(D) + pro.eps);
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = float((double(h[i]) * sc) * double(wq[i]));
    }
    const int jb = warp - rank * p.nbc;
    if (jb >= 0 && jb < p.nbc)
      q8k_block_warp(h, lane, nullptr, act_a + (size_t(c) * p.nbc + jb) * Q8A_REC,
                     act_b + (size_t(c) * p.nbc + jb) * Q8B_REC);
  }
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

  // unit u of this warp: tile (u / bpw) of the cluster's list, local block
  // warp + 8 * (u % bpw), ring slot u % R; the issue side walks them with
  // counters (lane 0 only)
  int is_i = 0, is_k = 0, is_s = 0;
  auto issue_next = [&]() {
    const int tile = cid + is_i * ncl;
    const int b = rank * p.nbc + warp + GX_WARPS * is_k;
    const GemvSeg& sg = p.seg[gx_seg_of(p, tile)];
    const uint32_t ub = uint32_t(unit_bytes(sg.type));
    uint64_t* bar = wb + is_s;
    mbar_expect_tx(bar, ub);
    bulk_copy_g2s(ring + size_t(is_s) * p.slot, sg.w + (size_t(tile - sg.tile_begin) * p.nb + b) * ub, ub, bar);
    if (++is_k == bpw) {
      is_k = 0;
      ++is_i;
    }
    if (++is_s == R) is_s = 0;
  };
  const int primed = n < R ? n : R;
  if (lane == 0) {
    for (int s = 0; s < R; ++s) mbar_init(wb + s, 1);
    for (int u = 0; u < primed; ++u) issue_next();
  }
  __syncwarp();
  pdl_wait();  // the activation records are written by the previous kernel
  // this CTA's activation records (blocks [rank * nbc, (rank + 1) * nbc) of
  // every column): computed by the prologue, or one bulk copy per column and
  // plane of the records the previous kernel wrote
  if (p.pro.mode != GEMV_PRO_NONE) {
    gx_prologue(p, act_a, act_b, rank, warp, lane);
    if (threadIdx.x == 0) {  // the wait below then passes at once
      mbar_init(&act_bar, 1);
      asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_u32(&act_bar)) : "memory");
    }
  } else if (threadIdx.x == 0) {
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
  int rs = 0;         // ring slot of the next unit consumed
  uint32_t rph = 0;   // its phase parity
  for (int i = 0; i < ntl; ++i) {
    const int tile = cid + i * ncl;
    const GemvSeg& sg = p.seg[gx_seg_of(p, tile)];
    const bool q4 = sg.type == TYPE_Q4_K;
    float* pbuf = prod + size_t(i & 1) * pstride;
    for (int k = 0; k < bpw; ++k) {
      const int u = i * bpw + k;
      if (ok && !mbar_wait_parity_sleep(wb + rs, rph, p.err)) ok = false;
      const int jb = warp + GX_WARPS * k;  // block inside this CTA's part
      if (ok) {
        const uint8_t* unit = ring + size_t(rs) * p.slot;
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
        if (ok && lane == 0) issue_next();
        if (ok) ++issued;
      }
      if (++rs == R) {
        rs = 0;
        rph ^= 1u;
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
        const int bstride = p.ncols * GX_PROD;  // floats between consecutive blocks' products
        for (int c = 0; c < p.ncols; ++c) {
          for (int kk = warp; kk < 9; kk += GX_WARPS) {
            float acc = 0.0f;
            const float* base = pb + (size_t(c) * 9 + kk) * 32 + lane;
            for (int r = 0; r < C; ++r) {  // blocks in row order: rank by rank
              const float* src = r == 0 ? base : cg::this_cluster().map_shared_rank(base, r);
              if (kk < 8) {
#pragma unroll 8
                for (int jb = 0; jb < p.nbc; ++jb) acc = __fadd_rn(acc, src[jb * bstride]);
              } else {
#pragma unroll 8
                for (int jb = 0; jb < p.nbc; ++jb) acc = __fsub_rn(acc, src[jb * bstride]);
              }
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

// ---- warp-per-tile form (rows of at most GW_MAX_NB blocks) -----------------
//
// A warp owns one (tile, column group) work item and walks the tile's nb
// blocks in order itself, the reference's nine accumulators of each of its
// columns in registers (LaneChain): no product buffer, no barrier, no chain
// phase.  Units stream through the warp's own ring of R slots (one bulk copy
// each, issued before griddepcontrol.wait for the first R units); the CTA's
// activation records (every column, every block) are staged once.  Work
// items go to warps round-robin over the CTAs first (item i -> CTA i mod
// grid), so a launch with few tiles still spreads over the SMs.
constexpr int GW_MAX_NB = 16;

__host__ __device__ inline size_t gw_smem_bytes(const GemvxParams& p) {
  return size_t(GX_WARPS) * p.R * p.slot + gx_act_bytes(p);
}

template <int NC>
__global__ void __launch_bounds__(GX_THREADS, 1) hc_gemvw_kernel(const __grid_constant__ GemvxParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[GX_WARPS * GX_MAX_R];
  __shared__ __align__(8) uint64_t act_bar;
  const int lane = int(threadIdx.x) & 31, warp = int(threadIdx.x) >> 5;
  pdl_trigger();
  const int R = p.R, nb = p.nb;
  const int ngroups = (p.ncols + NC - 1) / NC;  // column groups of NC columns
  const int nitems = p.total_tiles * ngroups;   // item = tile * ngroups + group
  const int gw = warp * int(gridDim.x) + int(blockIdx.x), nw = GX_WARPS * int(gridDim.x);
  const int nmine = gw < nitems ? (nitems - 1 - gw) / nw + 1 : 0;
  const int n = nmine * nb;  // this warp's units
  uint8_t* ring = smem + size_t(warp) * R * p.slot;
  uint8_t* act_a = smem + size_t(GX_WARPS) * R * p.slot;                          // [ncols][nb][288]
  uint8_t* act_b = act_a + ((p.planes & 1) ? size_t(p.ncols) * nb * Q8A_REC : 0);  // [ncols][nb][304]
  uint64_t* wb = bars + warp * R;

  // issue side (lane 0): unit (item, block b) into slot s
  int is_item = gw, is_tile = gw / ngroups, is_b = 0, is_s = 0;
  auto issue_next = [&]() {
    const GemvSeg& sg = p.seg[gx_seg_of(p, is_tile)];
    const uint32_t ub = uint32_t(unit_bytes(sg.type));
    uint64_t* bar = wb + is_s;
    mbar_expect_tx(bar, ub);
    bulk_copy_g2s(ring + size_t(is_s) * p.slot, sg.w + (size_t(is_tile - sg.tile_begin) * nb + is_b) * ub, ub, bar);
    if (++is_b == nb) {
      is_b = 0;
      is_item += nw;
      is_tile = is_item / ngroups;
    }
    if (++is_s == R) is_s = 0;
  };
  const int primed = n < R ? n : R;
  if (lane == 0) {
    for (int s = 0; s < R; ++s) mbar_init(wb + s, 1);
    for (int u = 0; u < primed; ++u) issue_next();
  }
  __syncwarp();
  pdl_wait();  // the activation records are written by the previous kernel
  if (p.pro.mode != GEMV_PRO_NONE) {
    gx_prologue(p, act_a, act_b, 0, warp, lane);
    if (threadIdx.x == 0) {
      mbar_init(&act_bar, 1);
      mbar_arrive(&act_bar);
    }
  } else if (threadIdx.x == 0) {
    mbar_init(&act_bar, 1);
    mbar_expect_tx(&act_bar, uint32_t(gx_act_bytes(p)));
    for (int c = 0; c < p.ncols; ++c) {
      const size_t rec0 = size_t(p.col0 + c) * nb;
      if (p.planes & 1)
        bulk_copy_g2s(act_a + size_t(c) * nb * Q8A_REC, p.q.a + rec0 * Q8A_REC, uint32_t(nb * Q8A_REC), &act_bar);
      if (p.planes & 2)
        bulk_copy_g2s(act_b + size_t(c) * nb * Q8B_REC, p.q.b + rec0 * Q8B_REC, uint32_t(nb * Q8B_REC), &act_bar);
    }
  }
  __syncthreads();
  bool ok = mbar_wait_parity(&act_bar, 0, p.err);
  int issued = primed, u = 0, rs = 0;
  uint32_t rph = 0;
  for (int it = 0; it < nmine; ++it) {
    const int item = gw + it * nw;
    const int tile = item / ngroups, c0 = (item - tile * ngroups) * NC;
    const GemvSeg& sg = p.seg[gx_seg_of(p, tile)];
    const bool q4 = sg.type == TYPE_Q4_K;
    LaneChain ch[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) ch[c].zero();
    for (int b = 0; b < nb; ++b, ++u) {
      if (ok && !mbar_wait_parity_sleep(wb + rs, rph, p.err)) ok = false;
      if (ok) {
        const uint8_t* unit = ring + size_t(rs) * p.slot;
        const SmemSrc src{reinterpret_cast<const uint4*>(unit) + lane,
                          reinterpret_cast<const uint16_t*>(unit + Q6K_DPLANE_OFFSET) + lane};
        if (q4) {
          const Q4KHeader hd = q4k_header(src.chunk(0));
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            if (c0 + c < p.ncols) {
              const uint8_t* rec = act_a + (size_t(c0 + c) * nb + b) * Q8A_REC;
              BlockInts bi;
              q4k_lanes(src, hd, rec, bi);
              const float d8 = *reinterpret_cast<const float*>(rec + Q8A_D);
              ch[c].add_block(bi, __fmul_rn(hd.d, d8), __fmul_rn(hd.dmin, d8), true);
            }
          }
        } else {
          const float dw = f16_bits_to_f32(src.dbits());
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            if (c0 + c < p.ncols) {
              const uint8_t* rec = act_b + (size_t(c0 + c) * nb + b) * Q8B_REC;
              BlockInts bi;
              q6k_lanes(src, rec, bi);
              ch[c].add_block(bi, __fmul_rn(dw, *reinterpret_cast<const float*>(rec + Q8B_D)), 0.0f, false);
            }
          }
        }
      }
      __syncwarp();  // every lane has read the slot: refill it
      if (u + R < n && ok) {
        if (lane == 0) issue_next();
        ++issued;
      }
      if (++rs == R) {
        rs = 0;
        rph ^= 1u;
      }
    }
    if (ok) {
      const int row = (tile - sg.tile_begin) * TILE + lane;
      if (row < sg.rows) {
#pragma unroll
        for (int c = 0; c < NC; ++c)
          if (c0 + c < p.ncols) sg.out[size_t(p.col0 + c0 + c) * sg.rows + row] = ch[c].total(q4);
      }
    }
  }
  if (!ok)
    for (int v = 0; v < issued; ++v) mbar_wait_parity(wb + (v % R), uint32_t(v / R) & 1u, nullptr);
}

// ---- tensor-core lane sums (Q4_K rows of at most 16 blocks, 2..8 columns) ----
//
// The warp-per-tile form with the integer lane sums of every column on
// mma.sync s8 m16n8k32.  The reference's lane l of a block (elements l,
// l + 8, l + 16, l + 24 of each 32-group) has the integer sum
//     aux32[l] = sum_g sc_g * dot_g,l       (sc_g: the 6-bit group scale).
// Split sc_g = 8 * hi_g + lo_g (3 bits each): q * lo_g and q * hi_g are at
// most 15 * 7 = 105, so the pre-scaled 4-bit values are int8 operands and
//     aux32[l] = D0 + 8 * D1,  D0 = sum_g dot(q * lo_g, q8), D1 = the same with hi_g,
// two 32-deep MMAs whose K runs over lane l's four elements of all eight
// groups (thread t's K slots are groups 2t and 2t + 1: exactly word l of quant
// pair t, low and high nibbles; the B fragment is the activation record's
// words of the same groups and lane).  Exact integers, so the f32 part --
// the reference's nine accumulators per (row, column), advanced per block in
// block order -- is the warp-per-tile form's, and the outputs are the same
// bit for bit.  A work item is one 16-row half of a tile (one m16 tile) and
// every column of the launch, so the weight-side work (unpacking, scaling)
// is shared by all columns; lane (g = lane / 4, t = lane % 4) holds rows
// g, g + 8 of the half and columns 2t, 2t + 1 (the m16n8 accumulator layout).
__device__ __forceinline__ uint32_t u4_word(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

constexpr int GT_MAX_SMEM = 110 * 1024;  // two CTAs per SM

__global__ void __launch_bounds__(GX_THREADS, 2) hc_gemvt_kernel(const __grid_constant__ GemvxParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[GX_WARPS * GX_MAX_R];
  __shared__ __align__(8) uint64_t act_bar;
  const int lane = int(threadIdx.x) & 31, warp = int(threadIdx.x) >> 5;
  const int g = lane >> 2, t = lane & 3;
  pdl_trigger();
  const int R = p.R, nb = p.nb, ncols = p.ncols;
  const int nitems = 2 * p.total_tiles;  // item = (tile, 16-row half), every column
  const int gw = warp * int(gridDim.x) + int(blockIdx.x), nw = GX_WARPS * int(gridDim.x);
  const int nmine = gw < nitems ? (nitems - 1 - gw) / nw + 1 : 0;
  const int n = nmine * nb;  // this warp's units
  uint8_t* ring = smem + size_t(warp) * R * p.slot;
  uint8_t* act_a = smem + size_t(GX_WARPS) * R * p.slot;                       // [ncols][nb][288]
  uint8_t* act_b = act_a + ((p.planes & 1) ? size_t(ncols) * nb * Q8A_REC : 0);  // written by the prologue only
  uint64_t* wb = bars + warp * R;

  int is_item = gw, is_b = 0, is_s = 0;
  auto issue_next = [&]() {
    const int tile = is_item >> 1;
    const GemvSeg& sg = p.seg[gx_seg_of(p, tile)];
    uint64_t* bar = wb + is_s;
    mbar_expect_tx(bar, uint32_t(Q4K_TILE_BLOCK_BYTES));
    bulk_copy_g2s(ring + size_t(is_s) * p.slot,
                  sg.w + (size_t(tile - sg.tile_begin) * nb + is_b) * Q4K_TILE_BLOCK_BYTES,
                  uint32_t(Q4K_TILE_BLOCK_BYTES), bar);
    if (++is_b == nb) {
      is_b = 0;
      is_item += nw;
    }
    if (++is_s == R) is_s = 0;
  };
  const int primed = n < R ? n : R;
  if (lane == 0) {
    for (int s = 0; s < R; ++s) mbar_init(wb + s, 1);
    for (int u = 0; u < primed; ++u) issue_next();
  }
  __syncwarp();
  pdl_wait();  // the activation records are written by the previous kernel
  if (p.pro.mode != GEMV_PRO_NONE) {
    gx_prologue(p, act_a, act_b, 0, warp, lane);
    if (threadIdx.x == 0) {
      mbar_init(&act_bar, 1);
      mbar_arrive(&act_bar);
    }
  } else if (threadIdx.x == 0) {
    mbar_init(&act_bar, 1);
    mbar_expect_tx(&act_bar, uint32_t(size_t(ncols) * nb * Q8A_REC));
    for (int c = 0; c < ncols; ++c) {
      const size_t rec0 = size_t(p.col0 + c) * nb;
      bulk_copy_g2s(act_a + size_t(c) * nb * Q8A_REC, p.q.a + rec0 * Q8A_REC, uint32_t(nb * Q8A_REC), &act_bar);
    }
  }
  __syncthreads();
  bool ok = mbar_wait_parity(&act_bar, 0, p.err);
  const bool bcol = g < ncols;                                  // B fragment column g
  const bool ccol0 = 2 * t < ncols, ccol1 = 2 * t + 1 < ncols;  // accumulator columns 2t, 2t + 1
  int issued = primed, u = 0, rs = 0;
  uint32_t rph = 0;
  for (int it = 0; it < nmine; ++it) {
    const int item = gw + it * nw, tile = item >> 1, r0 = 16 * (item & 1) + g;  // rows r0, r0 + 8
    const GemvSeg& sg = p.seg[gx_seg_of(p, tile)];
    LaneChain ch[4];  // pair 2i + cc: row r0 + 8i, column 2t + cc
#pragma unroll
    for (int k = 0; k < 4; ++k) ch[k].zero();
    for (int b = 0; b < nb; ++b, ++u) {
      if (ok && !mbar_wait_parity_sleep(wb + rs, rph, p.err)) ok = false;
      if (ok) {
        const uint8_t* unit = ring + size_t(rs) * p.slot;
        float dd[2], dm[2];
        uint32_t mnl[2], mnh[2], s0a[2], s1a[2], s0b[2], s1b[2];
        uint4 qlo[2], qhi[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int row = r0 + 8 * i;
          const Q4KHeader hd = q4k_header_hw(*reinterpret_cast<const uint4*>(unit + row * 16));
          dd[i] = hd.d;
          dm[i] = hd.dmin;
          mnl[i] = hd.mn_lo;
          mnh[i] = hd.mn_hi;
          const uint32_t sw = t < 2 ? hd.sc_lo : hd.sc_hi, sh = 16u * uint32_t(t & 1);
          const uint32_t sa = (sw >> sh) & 0xffu, sb = (sw >> (sh + 8u)) & 0xffu;  // groups 2t, 2t + 1
          s0a[i] = sa & 7u;
          s1a[i] = sa >> 3;
          s0b[i] = sb & 7u;
          s1b[i] = sb >> 3;
          qlo[i] = *reinterpret_cast<const uint4*>(unit + (1 + 2 * t) * 512 + row * 16);
          qhi[i] = *reinterpret_cast<const uint4*>(unit + (2 + 2 * t) * 512 + row * 16);
        }
        // B: column g's words of groups 2t (lanes 0..7) and 2t + 1
        uint4 bl0 = make_uint4(0, 0, 0, 0), bl1 = bl0, bh0 = bl0, bh1 = bl0;
        if (bcol) {
          const uint8_t* rec = act_a + (size_t(g) * nb + b) * Q8A_REC + 64 * t;
          bl0 = *reinterpret_cast<const uint4*>(rec);
          bl1 = *reinterpret_cast<const uint4*>(rec + 16);
          bh0 = *reinterpret_cast<const uint4*>(rec + 32);
          bh1 = *reinterpret_cast<const uint4*>(rec + 48);
        }
        // per (row, column) pair: d * d8, dmin * d8 and the min sum
        float pd[4], pm[4];
        int ms[4];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const bool cok = cc == 0 ? ccol0 : ccol1;
          const uint8_t* rec = act_a + (size_t(cok ? 2 * t + cc : 0) * nb + b) * Q8A_REC;
          const uint4 bs = *reinterpret_cast<const uint4*>(rec + Q8A_BS);
          const float d8 = *reinterpret_cast<const float*>(rec + Q8A_D);
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            pd[2 * i + cc] = __fmul_rn(dd[i], d8);
            pm[2 * i + cc] = __fmul_rn(dm[i], d8);
            int m = __dp2a_lo(int(bs.x), int(mnl[i]), 0);
            m = __dp2a_hi(int(bs.y), int(mnl[i]), m);
            m = __dp2a_lo(int(bs.z), int(mnh[i]), m);
            ms[2 * i + cc] = __dp2a_hi(int(bs.w), int(mnh[i]), m);
          }
        }
#pragma unroll
        for (int l = 0; l < 8; ++l) {
          const uint32_t b0 = u4_word(l < 4 ? bl0 : bl1, l & 3), b1 = u4_word(l < 4 ? bh0 : bh1, l & 3);
          const uint32_t w0 = u4_word(l < 4 ? qlo[0] : qhi[0], l & 3);
          const uint32_t w1 = u4_word(l < 4 ? qlo[1] : qhi[1], l & 3);
          const uint32_t lo0 = w0 & 0x0f0f0f0fu, lo1 = w1 & 0x0f0f0f0fu;
          const uint32_t hi0 = (w0 >> 4) & 0x0f0f0f0fu, hi1 = (w1 >> 4) & 0x0f0f0f0fu;
          int d0[4], d1[4];
          mma_k32(d0, lo0 * s0a[0], lo1 * s0a[1], hi0 * s0b[0], hi1 * s0b[1], b0, b1);
          mma_k32(d1, lo0 * s1a[0], lo1 * s1a[1], hi0 * s1b[0], hi1 * s1b[1], b0, b1);
#pragma unroll
          for (int r = 0; r < 4; ++r)  // r: (row r0 + 8 (r >> 1), column 2t + (r & 1)) = pair r
            ch[r].s[l] = __fadd_rn(ch[r].s[l], __fmul_rn(pd[r], float(d0[r] + 8 * d1[r])));
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) ch[k].m = __fsub_rn(ch[k].m, __fmul_rn(pm[k], float(ms[k])));
      }
      __syncwarp();  // every lane has read the slot: refill it
      if (u + R < n && ok) {
        if (lane == 0) issue_next();
        ++issued;
      }
      if (++rs == R) {
        rs = 0;
        rph ^= 1u;
      }
    }
    if (ok) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int row = (tile - sg.tile_begin) * TILE + r0 + 8 * i;
        if (row < sg.rows) {
          if (ccol0) sg.out[size_t(p.col0 + 2 * t) * sg.rows + row] = ch[2 * i].total(true);
          if (ccol1) sg.out[size_t(p.col0 + 2 * t + 1) * sg.rows + row] = ch[2 * i + 1].total(true);
        }
      }
    }
  }
  if (!ok)
    for (int v = 0; v < issued; ++v) mbar_wait_parity(wb + (v % R), uint32_t(v / R) & 1u, nullptr);
}

// ---- relay form (long rows: nb = 8 * NBP blocks) ------------------------------
//
// One CTA per (tile, column): warp w owns blocks [w * NBP, (w + 1) * NBP) of
// the row, streams its NBP units through its ring and parks the reference's
// nine f32 products of each block (d * aux32[l], dmin * sumi) in its own
// shared-memory slab prod[w][NBP][9][32] (the block loop stays rolled: one
// copy of the block decode keeps the kernel inside the instruction cache).
// The nine accumulators then pass from warp to warp in block order through
// shared memory (relay[w][9][32], one mbarrier per hop): warp w adds its
// products to what warp w - 1 handed over, exactly the reference's
// sequential block loop, and warp 7 writes the row total.  Only the hops are
// serial; the integer work of all 8 * NBP blocks runs in parallel.
constexpr int GR_PARTS = GX_WARPS;

// activation records: the CTA's column only, or every column when the
// prologue computes them (it norms the whole launch's input)
__host__ __device__ inline int gr_act_cols(const GemvxParams& p) { return p.pro.mode != GEMV_PRO_NONE ? p.ncols : 1; }
__host__ __device__ inline size_t gr_act_bytes(const GemvxParams& p) {
  return size_t(gr_act_cols(p)) * p.nb * (((p.planes & 1) ? Q8A_REC : 0) + ((p.planes & 2) ? Q8B_REC : 0));
}
__host__ __device__ inline size_t gr_smem_bytes(const GemvxParams& p) {
  return size_t(GR_PARTS) * p.R * p.slot + gr_act_bytes(p) + size_t(GR_PARTS) * GX_PROD * sizeof(float) +
         size_t(GR_PARTS) * (p.nb / (GR_PARTS * p.C)) * GX_PROD * sizeof(float);
}

// The relay's hop from the last warp of one CTA to the first warp of the
// next CTA of its cluster: that CTA's relay words are written through
// distributed shared memory, then each lane arrives on the CTA's hop
// barrier with release semantics at cluster scope.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t* bar, int rank) {
  asm volatile(
      "{ .reg .b32 ra; mapa.shared::cluster.u32 ra, %0, %1; "
      "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra]; }" ::"r"(smem_u32(bar)),
      "r"(rank)
      : "memory");
}
// Bounded wait whose completion also acquires what other CTAs of the
// cluster released before arriving (same bound and status as mbar_wait_parity).
__device__ __forceinline__ bool mbar_wait_parity_cluster(uint64_t* bar, uint32_t parity, int* err) {
  unsigned long long t0 = 0;
  for (int it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3; "
        "selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(SLEEP_HINT_NS)
        : "memory");
    if (ok) return true;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (it == 0) {
      t0 = t;
    } else if (t - t0 > WAIT_LIMIT_NS) {
      if (err) atomicExch(err, DEVICE_ERR_TIMEOUT);
      return false;
    }
  }
}
constexpr int GR_MAX_SMEM = 220 * 1024;

template <int NBP>
__global__ void __launch_bounds__(GX_THREADS, 1) hc_gemvr_kernel(const __grid_constant__ GemvxParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[GX_WARPS * GX_MAX_R];
  __shared__ __align__(8) uint64_t act_bar;
  __shared__ __align__(8) uint64_t hop[GR_PARTS];
  const int lane = int(threadIdx.x) & 31, warp = int(threadIdx.x) >> 5;
  pdl_trigger();
  const int R = p.R, nb = p.nb, C = p.C;
  const int cid = int(blockIdx.x) / C, rank = int(blockIdx.x) - cid * C;  // a cluster of C CTAs per (tile, column)
  const int tile = cid / p.ncols, c = cid - tile * p.ncols;
  const GemvSeg& sg = p.seg[gx_seg_of(p, tile)];
  const bool q4 = sg.type == TYPE_Q4_K;
  const uint32_t ub = uint32_t(unit_bytes(sg.type));
  const uint8_t* wtile = sg.w + size_t(tile - sg.tile_begin) * nb * ub;
  uint8_t* ring = smem + size_t(warp) * R * p.slot;
  const int acols = gr_act_cols(p);
  uint8_t* act_a = smem + size_t(GR_PARTS) * R * p.slot;                      // [acols][nb][288]
  uint8_t* act_b = act_a + ((p.planes & 1) ? size_t(acols) * nb * Q8A_REC : 0);  // [acols][nb][304]
  float* relay = reinterpret_cast<float*>(act_a + gr_act_bytes(p));  // [8][9][32]
  float* prod = relay + GR_PARTS * GX_PROD + size_t(warp) * NBP * GX_PROD + lane;  // this warp's [NBP][9][32]
  uint64_t* wb = bars + warp * R;
  const int b0 = (rank * GR_PARTS + warp) * NBP;
  if (lane == 0) {
    for (int s = 0; s < R; ++s) mbar_init(wb + s, 1);
    for (int k = 0; k < R && k < NBP; ++k) {
      mbar_expect_tx(wb + k, ub);
      bulk_copy_g2s(ring + size_t(k) * p.slot, wtile + size_t(b0 + k) * ub, ub, wb + k);
    }
  }
  if (threadIdx.x == 0)
    for (int w = 0; w < GR_PARTS; ++w) mbar_init(&hop[w], 32);
  __syncwarp();
  pdl_wait();  // the activation records are written by the previous kernel
  if (p.pro.mode != GEMV_PRO_NONE) {
    gx_prologue(p, act_a, act_b, 0, warp, lane);  // every column (row width 2048: one block per warp)
    if (threadIdx.x == 0) {
      mbar_init(&act_bar, 1);
      mbar_arrive(&act_bar);
    }
  } else if (threadIdx.x == 0) {
    mbar_init(&act_bar, 1);
    mbar_expect_tx(&act_bar, uint32_t(gr_act_bytes(p)));
    const size_t rec0 = size_t(p.col0 + c) * nb;
    if (p.planes & 1) bulk_copy_g2s(act_a, p.q.a + rec0 * Q8A_REC, uint32_t(nb * Q8A_REC), &act_bar);
    if (p.planes & 2) bulk_copy_g2s(act_b, p.q.b + rec0 * Q8B_REC, uint32_t(nb * Q8B_REC), &act_bar);
  }
  __syncthreads();
  // the hop barriers are initialized before another CTA of the cluster may
  // arrive on them (waited for before the relay)
  if (C > 1) asm volatile("barrier.cluster.arrive.release;" ::: "memory");
  bool ok = mbar_wait_parity(&act_bar, 0, p.err);
  const int ac = acols > 1 ? c : 0;  // this CTA's column among the staged records
  act_a += size_t(ac) * nb * Q8A_REC;
  act_b += size_t(ac) * nb * Q8B_REC;
  int issued = R < NBP ? R : NBP;
  int rs = 0;
  uint32_t rph = 0;
#pragma unroll 1
  for (int k = 0; k < NBP; ++k) {
    if (ok && !mbar_wait_parity_sleep(wb + rs, rph, p.err)) ok = false;
    const int b = b0 + k;
    if (ok) {
      const uint8_t* unit = ring + size_t(rs) * p.slot;
      const SmemSrc src{reinterpret_cast<const uint4*>(unit) + lane,
                        reinterpret_cast<const uint16_t*>(unit + Q6K_DPLANE_OFFSET) + lane};
      BlockInts bi;
      float d, dm = 0.0f;
      if (q4) {
        const Q4KHeader hd = q4k_header(src.chunk(0));
        const uint8_t* rec = act_a + size_t(b) * Q8A_REC;
        q4k_lanes(src, hd, rec, bi);
        const float d8 = *reinterpret_cast<const float*>(rec + Q8A_D);
        d = __fmul_rn(hd.d, d8);
        dm = __fmul_rn(hd.dmin, d8);
      } else {
        const uint8_t* rec = act_b + size_t(b) * Q8B_REC;
        q6k_lanes(src, rec, bi);
        d = __fmul_rn(f16_bits_to_f32(src.dbits()), *reinterpret_cast<const float*>(rec + Q8B_D));
      }
      float* pk = prod + k * GX_PROD;
#pragma unroll
      for (int l = 0; l < 8; ++l) pk[l * 32] = __fmul_rn(d, float(bi.aux[l]));
      pk[8 * 32] = __fmul_rn(dm, float(bi.msum));
    }
    __syncwarp();  // every lane has read the slot: refill it
    if (k + R < NBP && ok) {
      if (lane == 0) {
        mbar_expect_tx(wb + rs, ub);
        bulk_copy_g2s(ring + size_t(rs) * p.slot, wtile + size_t(b + R) * ub, ub, wb + rs);
      }
      ++issued;
    }
    if (++rs == R) {
      rs = 0;
      rph ^= 1u;
    }
  }
  if (C > 1) asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
  // the relay: the accumulators after blocks 0 .. b0 - 1 come from the
  // previous warp (of this CTA, or the last warp of the previous rank)
  float acc[9];
#pragma unroll
  for (int l = 0; l < 9; ++l) acc[l] = 0.0f;
  if (warp > 0 || rank > 0) {
    if (ok && !(warp == 0 ? mbar_wait_parity_cluster(&hop[0], 0, p.err) : mbar_wait_parity_sleep(&hop[warp], 0, p.err)))
      ok = false;
#pragma unroll
    for (int l = 0; l < 9; ++l) acc[l] = relay[(warp * 9 + l) * 32 + lane];
  }
#pragma unroll
  for (int k = 0; k < NBP; ++k) {  // each lane reads back only its own words
    const float* pk = prod + k * GX_PROD;
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[l] = __fadd_rn(acc[l], pk[l * 32]);
    if (q4) acc[8] = __fsub_rn(acc[8], pk[8 * 32]);
  }
  if (warp + 1 < GR_PARTS) {
#pragma unroll
    for (int l = 0; l < 9; ++l) relay[((warp + 1) * 9 + l) * 32 + lane] = acc[l];
    mbar_arrive(&hop[warp + 1]);  // each lane releases its own words
  } else if (rank + 1 < C) {  // to the first warp of the next rank
    float* dst = cg::this_cluster().map_shared_rank(relay, rank + 1);
#pragma unroll
    for (int l = 0; l < 9; ++l) dst[l * 32 + lane] = acc[l];
    mbar_arrive_remote(&hop[0], rank + 1);
  } else if (ok) {
    float t = 0.0f;
#pragma unroll
    for (int l = 0; l < 8; ++l) t = __fadd_rn(t, acc[l]);
    const float v = q4 ? __fadd_rn(acc[8], t) : t;
    const int row = (tile - sg.tile_begin) * TILE + lane;
    if (row < sg.rows) sg.out[size_t(p.col0 + c) * sg.rows + row] = v;
  }
  if (!ok)
    for (int v = 0; v < issued; ++v) mbar_wait_parity(wb + (v % R), uint32_t(v / R) & 1u, nullptr);
  // no CTA leaves while another may still write its shared memory
  if (C > 1) {
    asm volatile("barrier.cluster.arrive.release;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
  }
}

}  // namespace

// HPC_GEMVX_FORM = w | r | x pins every launch that form takes to the
// warp-per-tile, relay or split (cluster) form, for comparing them; unset,
// the planners choose.
static char gemvx_form() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("HPC_GEMVX_FORM");
    v = e && (e[0] == 'w' || e[0] == 'r' || e[0] == 'x' || e[0] == 't') ? e[0] : 0;
  }
  return char(v);
}

int gemvx_plan(GemvxParams& p, int sms) {
  // ring slot: the largest unit among the launch's weights
  p.slot = 0;
  p.planes = 0;
  for (int i = 0; i < p.nseg; ++i) {
    p.slot = max(p.slot, unit_bytes(p.seg[i].type));
    p.planes |= p.seg[i].type == TYPE_Q4_K ? 1 : 2;
  }
  if (p.pro.mode != GEMV_PRO_NONE) {
    // the prologue writes both planes, and needs the whole width-2048 row
    // (one 256-block per warp) in one CTA
    if (p.K != GEMV_PRO_D) return -1;
    p.planes = 3;
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
      // (ties: more bytes in flight; two CTAs per SM win equal bytes -- twice
      // the warps to hide the shared-memory and barrier latencies)
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

// Warp-per-tile plan: columns per warp (returned) -- the fewest for which
// the work items fit two rounds of the launch's warps -- and the deepest
// ring that fits; returns the grid size via *grid (0: not this form, also
// for launches of few work items per SM).
int gemvw_plan(GemvxParams& p, int sms, int* grid, bool any_size) {
  *grid = 0;
  if (p.nb > GW_MAX_NB || p.ncols < 1 || p.ncols > GEMVX_MAX_COLS) return 0;
  p.slot = 0;
  p.planes = 0;
  for (int i = 0; i < p.nseg; ++i) {
    p.slot = max(p.slot, unit_bytes(p.seg[i].type));
    p.planes |= p.seg[i].type == TYPE_Q4_K ? 1 : 2;
  }
  if (p.pro.mode != GEMV_PRO_NONE) {
    if (p.K != GEMV_PRO_D) return 0;
    p.planes = 3;
  }
  p.C = 1;
  p.nbc = p.nb;
  int nc = 1;
  while (nc < p.ncols && p.total_tiles * ((p.ncols + nc - 1) / nc) > 2 * GX_WARPS * sms) nc *= 2;
  if (nc > p.ncols) nc = p.ncols <= 1 ? 1 : p.ncols <= 2 ? 2 : p.ncols <= 4 ? 4 : 8;
  for (p.R = GX_MAX_R; p.R >= 1; --p.R)
    if (gw_smem_bytes(p) <= size_t(GEMV_MAX_SMEM)) break;
  if (p.R < 1) return 0;
  const int nitems = p.total_tiles * ((p.ncols + nc - 1) / nc);
  // a launch of few items runs each item on a single warp's serial block
  // loop, and the split form spreads it wider: measured, the split form is
  // faster below 4 one-column items per SM (config 1: 512 items, 6.5 vs
  // 7.6 us) and below 2 items per SM with more columns
  if (nitems < (p.ncols == 1 ? 4 : 2) * sms && !any_size) return 0;
  *grid = min(sms, nitems);
  p.err = device_status_word();
  return nc <= 1 ? 1 : nc <= 2 ? 2 : nc <= 4 ? 4 : 8;
}

// Tensor-core lane-sum plan: every segment Q4_K, 2..8 columns, rows of at
// most GW_MAX_NB blocks, at least 2 tiles per SM (fewer leave most SMs to a
// single warp: the other forms split those finer); one warp per 16-row half
// tile; the deepest ring that fits.  Returns the grid size (0: not this form).
static int gemvt_plan(GemvxParams& p, int sms, bool any_size) {
  if (p.nb > GW_MAX_NB || p.ncols < 2 || p.ncols > 8) return 0;
  if (p.total_tiles < 2 * sms && !any_size) return 0;
  for (int i = 0; i < p.nseg; ++i)
    if (p.seg[i].type != TYPE_Q4_K) return 0;
  p.slot = int(Q4K_TILE_BLOCK_BYTES);
  p.planes = 1;
  if (p.pro.mode != GEMV_PRO_NONE) {
    if (p.K != GEMV_PRO_D) return 0;
    p.planes = 3;
  }
  p.C = 1;
  p.nbc = p.nb;
  for (p.R = GX_MAX_R; p.R >= 1; --p.R)
    if (gw_smem_bytes(p) <= size_t(GT_MAX_SMEM)) break;
  if (p.R < 1) return 0;
  p.err = device_status_word();
  return min(2 * sms, 2 * p.total_tiles);
}

// Relay plan: rows of 16, 32 or 64 blocks, no prologue, every segment one
// type; the deepest ring (at most the blocks per part) that fits.  Returns
// the blocks per part (0: not this form).
static int gemvr_plan(GemvxParams& p, int sms) {
  if (p.nb % GR_PARTS != 0) return 0;
  if (p.pro.mode != GEMV_PRO_NONE && p.K != GEMV_PRO_D) return 0;
  // a CTA pair per (tile, column) when one CTA each would leave half the SMs idle
  p.C = p.total_tiles * p.ncols * 2 <= sms && p.nb % (2 * GR_PARTS) == 0 && p.nb / (2 * GR_PARTS) >= 2 ? 2 : 1;
  const int nbp = p.nb / (GR_PARTS * p.C);
  if (nbp != 1 && nbp != 2 && nbp != 4 && nbp != 8) return 0;
  p.slot = 0;
  p.planes = 0;
  for (int i = 0; i < p.nseg; ++i) {
    p.slot = max(p.slot, unit_bytes(p.seg[i].type));
    p.planes |= p.seg[i].type == TYPE_Q4_K ? 1 : 2;
  }
  if (p.pro.mode != GEMV_PRO_NONE) p.planes = 3;  // the prologue writes both planes
  p.nbc = p.nb / p.C;
  for (p.R = min(GX_MAX_R, nbp); p.R >= 1; --p.R)
    if (gr_smem_bytes(p) <= size_t(GR_MAX_SMEM)) break;
  if (p.R < 1) return 0;
  p.err = device_status_word();
  return nbp;
}

template <int NBP>
static cudaError_t launch_r(const GemvxParams& p, cudaStream_t st) {
  const size_t smem = gr_smem_bytes(p);
  static std::atomic<uint64_t> attr_set{0};
  const cudaError_t ea = once_per_current_device(attr_set, [] {
    return cudaFuncSetAttribute(hc_gemvr_kernel<NBP>, cudaFuncAttributeMaxDynamicSharedMemorySize, GR_MAX_SMEM);
  });
  if (ea != cudaSuccess) return ea;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(p.total_tiles * p.ncols * p.C));
  cfg.blockDim = dim3(GX_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int na = 1;
  if (p.C > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = unsigned(p.C);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    na = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, hc_gemvr_kernel<NBP>, p);
}

template <int NC>
static cudaError_t launch_w(const GemvxParams& p, int grid, cudaStream_t st) {
  const size_t smem = gw_smem_bytes(p);
  static std::atomic<uint64_t> attr_set{0};
  const cudaError_t ea = once_per_current_device(attr_set, [] {
    return cudaFuncSetAttribute(hc_gemvw_kernel<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_MAX_SMEM);
  });
  if (ea != cudaSuccess) return ea;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(GX_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, hc_gemvw_kernel<NC>, p);
}

static cudaError_t launch_t(const GemvxParams& p, int grid, cudaStream_t st) {
  static std::atomic<uint64_t> attr_set{0};
  const cudaError_t ea = once_per_current_device(attr_set, [] {
    return cudaFuncSetAttribute(hc_gemvt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GT_MAX_SMEM);
  });
  if (ea != cudaSuccess) return ea;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(GX_THREADS);
  cfg.dynamicSmemBytes = gw_smem_bytes(p);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, hc_gemvt_kernel, p);
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
  const char form = gemvx_form();
  // 2..8 columns of Q4_K rows: the integer lane sums on the tensor cores
  if (form == 0 || form == 't') {
    GemvxParams t = p;
    const int tgrid = gemvt_plan(t, sm_count(), form == 't');
    if (tgrid > 0) {
      p = t;
      return launch_t(p, tgrid, st);
    }
  }
  if (form == 0 || form == 'w') {
    int wgrid = 0;
    const int nc = gemvw_plan(p, sm_count(), &wgrid, form == 'w');
    if (nc > 0 && wgrid > 0) {
      if (nc == 1) return launch_w<1>(p, wgrid, st);
      if (nc == 2) return launch_w<2>(p, wgrid, st);
      if (nc == 4) return launch_w<4>(p, wgrid, st);
      return launch_w<8>(p, wgrid, st);
    }
  }
  // the relay form serves rows of 16+ blocks (and, pinned, rows of 8)
  if (form == 0 || form == 'r') {
    GemvxParams r = p;
    const int nbp = form == 'r' || p.nb > GW_MAX_NB ? gemvr_plan(r, sm_count()) : 0;
    if (nbp == 1) return launch_r<1>(r, st);
    if (nbp == 2) return launch_r<2>(r, st);
    if (nbp == 4) return launch_r<4>(r, st);
    if (nbp == 8) return launch_r<8>(r, st);
  }
  const int grid = gemvx_plan(p, sm_count());
  if (grid <= 0) return cudaErrorInvalidValue;
  if (p.ncols <= 1) return launch_x<1>(p, grid, st);
  if (p.ncols <= 2) return launch_x<2>(p, grid, st);
  if (p.ncols <= 4) return launch_x<4>(p, grid, st);
  return launch_x<8>(p, grid, st);
}

}  // namespace hc
