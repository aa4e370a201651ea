// hc_gemm_tc.cu -- Q4_K / Q6_K x Q8_K matmul on the tensor cores for wide
// inputs (M >= TC_MIN_COLS columns): prefill and the M = 64 LM head, where the
// product is a dense contraction rather than a weight stream.
//
// Same arithmetic as the GEMV (hc_gemv_body.cuh, i.e. vec_dot_q4_k_q8_k /
// vec_dot_q6_k_q8_k, lib.rs:2117-2172 / 1924-1968): the integer sum of every
// (row, column, sub-block) is exact, then scaled by the sub-block's integer
// scale, summed over the block in int32, and combined with d, dmin and the
// activation's d in f32 once per 256-block.
//
// Why mma.sync (s8, int32 accumulators in registers) and not tcgen05: the
// K-quant scales are per row and per 32- (Q4_K) or 16-element (Q6_K)
// sub-block, small integers that must multiply the exact sub-block sums
// before they are added.  With register accumulators that is one integer
// multiply-add per accumulator after each MMA; tcgen05's TMEM accumulators
// would need a round trip per K = 32 step, and its block-scaled kinds take
// only power-of-two style scale formats.
//
// Decomposition: a CTA of 8 warps covers 4 weight tiles (128 rows) x 64
// columns; warp w takes tile w % 4 and columns 32 (w / 4) .. + 31 as 2 x 4
// m16n8 accumulator tiles.  Per 256-block the CTA stages its 4 weight units
// (the row-tile layout of hc_common.cuh, unchanged) and its 64 columns' Q8_K
// records with cp.async into one of two shared-memory stages, so block b + 1
// streams in while block b is computed.  The records are staged at a
// 304-byte stride, which keeps the B-fragment loads of the eight columns in
// distinct banks.  Launches of fewer CTAs than two per SM (the 2048-row
// projections) split K in two halves over grid.z, whose partials are added
// atomically into a zeroed output: with exactly two addends the sum does not
// depend on their order.  The block products themselves are hc_mma.cuh's:
// the row-tile layout's words are directly the A fragments, the record words
// the B fragments, so no repack is needed.
#include "hc_bulk.cuh"
#include "hc_common.cuh"
#include "hc_kernels.cuh"
#include "hc_mma.cuh"

namespace hc {

constexpr int TC_WARPS = 8;
constexpr int TC_THREADS = 32 * TC_WARPS;
constexpr int TC_TILES = 4;   // weight tiles (32 rows) per CTA
constexpr int TC_COLS = 64;   // columns per CTA

struct TcParams {
  const uint8_t* w;    // tile layout
  const uint8_t* act;  // the Q8_K record plane this type reads (A for Q4_K, B for Q6_K), [col][nb]
  float* out;          // out[col * rows + row]
  int rows, tiles, nb, ncols, col0;
  int ksplit;          // 1, or 2: grid.z halves of K, atomically added into a zeroed out
};

template <int TYPE>
struct TcType {
  static constexpr int UB = TYPE == TYPE_Q4_K ? 4608 : 6720;
  static constexpr int REC = TYPE == TYPE_Q4_K ? Q8A_REC : Q8B_REC;
  // staged record stride: 304 bytes (76 words) for both planes puts the
  // eight columns' B-fragment words in distinct banks (288 would map
  // columns g and g + 4 onto the same ones)
  static constexpr int SREC = 304;
  static constexpr int STAGE = TC_TILES * UB + TC_COLS * SREC;
};

template <int TYPE>
__global__ void __launch_bounds__(TC_THREADS, 2) hc_gemm_tc_kernel(const __grid_constant__ TcParams p) {
  using T = TcType<TYPE>;
  extern __shared__ __align__(16) uint8_t smem[];
  const int tile0 = int(blockIdx.x) * TC_TILES, col0 = p.col0 + int(blockIdx.y) * TC_COLS;
  const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31), g = lane >> 2, t = lane & 3;
  const int wt = warp & 3, wh = warp >> 2;
  // Tiles past the end and columns past ncols are read clamped (never out of
  // the buffers) and not stored.
  auto issue = [&](int b, uint8_t* st) {
    for (int i = int(threadIdx.x); i < TC_TILES * T::UB / 16; i += TC_THREADS) {
      const int u = i / (T::UB / 16), o = i % (T::UB / 16);
      const int tile = min(tile0 + u, p.tiles - 1);
      cp_async16(st + u * T::UB + o * 16, p.w + (size_t(tile) * p.nb + b) * T::UB + o * 16);
    }
    for (int i = int(threadIdx.x); i < TC_COLS * T::REC / 16; i += TC_THREADS) {
      const int c = i / (T::REC / 16), o = i % (T::REC / 16);
      const int col = min(col0 + c, p.col0 + p.ncols - 1);
      cp_async16(st + TC_TILES * T::UB + c * T::SREC + o * 16, p.act + (size_t(col) * p.nb + b) * T::REC + o * 16);
    }
    cp_async_commit();
  };
  float acc[2][4][4];
#pragma unroll
  for (int mg = 0; mg < 2; ++mg)
#pragma unroll
    for (int ng = 0; ng < 4; ++ng)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[mg][ng][r] = 0.0f;
  // K range of this CTA: all blocks, or one half (ksplit 2)
  const int kb0 = int(blockIdx.z) * (p.nb / p.ksplit), kb1 = kb0 + p.nb / p.ksplit;
  issue(kb0, smem);
  for (int b = kb0; b < kb1; ++b) {
    if (b + 1 < kb1) {
      issue(b + 1, smem + ((b + 1 - kb0) & 1) * T::STAGE);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const uint8_t* st = smem + ((b - kb0) & 1) * T::STAGE;
    tc_block<TYPE, 4>(st + wt * T::UB, st + TC_TILES * T::UB + (32 * wh) * T::SREC, T::SREC, acc, g, t);
    __syncthreads();  // every warp is done with this stage before it is refilled
  }
  const int tile = tile0 + wt;
  if (tile >= p.tiles) return;
#pragma unroll
  for (int mg = 0; mg < 2; ++mg)
#pragma unroll
    for (int ng = 0; ng < 4; ++ng)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int row = tile * TILE + 16 * mg + g + 8 * (r >> 1);
        const int col = col0 + 32 * wh + 8 * ng + 2 * t + (r & 1);
        if (row < p.rows && col < p.col0 + p.ncols) {
          // two halves: a + b is the same sum in either order, so the
          // result stays deterministic
          if (p.ksplit == 1) p.out[size_t(col) * p.rows + row] = acc[mg][ng][r];
          else atomicAdd(p.out + size_t(col) * p.rows + row, acc[mg][ng][r]);
        }
      }
}

template <int TYPE>
static cudaError_t launch_tc(const TcParams& p, cudaStream_t st) {
  const size_t smem = 2 * size_t(TcType<TYPE>::STAGE);
  static std::atomic<uint64_t> attr{0};
  const cudaError_t ea = once_per_current_device(attr, [smem] {
    return cudaFuncSetAttribute(hc_gemm_tc_kernel<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  });
  if (ea != cudaSuccess) return ea;
  const dim3 grid(unsigned((p.tiles + TC_TILES - 1) / TC_TILES), unsigned((p.ncols + TC_COLS - 1) / TC_COLS),
                  unsigned(p.ksplit));
  if (p.ksplit > 1) {
    cudaError_t e = cudaMemsetAsync(p.out + size_t(p.col0) * p.rows, 0, sizeof(float) * size_t(p.ncols) * p.rows, st);
    if (e != cudaSuccess) return e;
  }
  hc_gemm_tc_kernel<TYPE><<<grid, TC_THREADS, smem, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_gemm_tc(const GemvSeg& seg, int nb, const Q8Buf& q, int col0, int ncols, cudaStream_t st) {
  if (seg.type == TYPE_Q4_K && gemm_t5_enabled()) return launch_gemm_t5(seg, nb, q, col0, ncols, st);
  TcParams p;
  p.w = seg.w;
  p.out = seg.out;
  p.rows = seg.rows;
  p.tiles = (seg.rows + TILE - 1) / TILE;
  p.nb = nb;
  p.ncols = ncols;
  p.col0 = col0;
  // fewer CTAs than two per SM (narrow outputs: the 2048-row projections)
  // and an even block count: split K in two
  const int ctas = ((p.tiles + TC_TILES - 1) / TC_TILES) * ((ncols + TC_COLS - 1) / TC_COLS);
  p.ksplit = (ctas < 2 * sm_count() && nb % 2 == 0) ? 2 : 1;
  if (seg.type == TYPE_Q4_K) {
    p.act = q.a;
    return launch_tc<TYPE_Q4_K>(p, st);
  }
  p.act = q.b;
  return launch_tc<TYPE_Q6_K>(p, st);
}

}  // namespace hc
