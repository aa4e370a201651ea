// hc_repack.cu -- GGUF block layout -> row-tile layout (see hc_common.cuh),
// and the inverse dequantization used to prove the repack bit-exact.
//
// Dequantization follows dequantize_q4_k (lib.rs:1630-1664):
//   y = (d*sc)*q - dmin*m
// and dequantize_q6_k (lib.rs:1709-1744):
//   y = (d*sc)*(q-32)
// with every product and difference rounded on its own (__fmul_rn/__fsub_rn),
// as the Rust code never fuses them.
#include "hc_bulk.cuh"
#include "hc_common.cuh"
#include "hc_kernels.cuh"
#include "hc_unpack.cuh"

namespace hc {

// ---- repack: one thread per (row, block) -----------------------------------

__global__ void hc_repack_q4k_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int rows,
                                  int rows_pad, int nb) {
  const size_t t = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
  if (t >= size_t(rows_pad) * nb) return;
  const int row = int(t / nb), b = int(t % nb);
  const int tile = row / TILE, lane = row % TILE;
  uint8_t blk[144];
  if (row < rows) {
    const uint8_t* s = src + (size_t(row) * nb + b) * 144;
    for (int i = 0; i < 144; ++i) blk[i] = s[i];
  } else {
    for (int i = 0; i < 144; ++i) blk[i] = 0;
  }
  uint8_t* out = dst + (size_t(tile) * nb + b) * Q4K_TILE_BLOCK_BYTES + size_t(lane) * 16;
  uint32_t w[4];
  for (int k = 0; k < 4; ++k) w[k] = blk[4 * k] | (blk[4 * k + 1] << 8) | (blk[4 * k + 2] << 16) | (uint32_t(blk[4 * k + 3]) << 24);
  *reinterpret_cast<uint4*>(out) = make_uint4(w[0], w[1], w[2], w[3]);
  const uint8_t* qs = blk + 16;
  for (int c = 0; c < 8; ++c) {
    const int p = c >> 1;
    for (int k = 0; k < 4; ++k) {
      const int l = 4 * (c & 1) + k;
      const int o = 32 * p + l;
      w[k] = qs[o] | (qs[o + 8] << 8) | (qs[o + 16] << 16) | (uint32_t(qs[o + 24]) << 24);
    }
    *reinterpret_cast<uint4*>(out + size_t(1 + c) * 16 * TILE) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__device__ __forceinline__ uint32_t q6_value(const uint8_t* blk, int e) {
  const int h = e >> 7, r = e & 127;
  const uint8_t lq = blk[64 * h + (r & 63)];
  const uint32_t lo = (r < 64) ? (lq & 0x0f) : (lq >> 4);
  const uint32_t hi = (blk[128 + 32 * h + (r & 31)] >> (2 * (r >> 5))) & 3;
  return lo | (hi << 4);
}

__device__ __forceinline__ int q6_elem(int s, int j, int i) {
  const int off[4] = {0, 8, 1, 9};
  return 16 * s + 2 * j + off[i];
}

__global__ void hc_repack_q6k_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int rows,
                                  int rows_pad, int nb) {
  const size_t t = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
  if (t >= size_t(rows_pad) * nb) return;
  const int row = int(t / nb), b = int(t % nb);
  const int tile = row / TILE, lane = row % TILE;
  uint8_t blk[210];
  if (row < rows) {
    const uint8_t* s = src + (size_t(row) * nb + b) * 210;
    for (int i = 0; i < 210; ++i) blk[i] = s[i];
  } else {
    for (int i = 0; i < 210; ++i) blk[i] = 0;
  }
  uint8_t* base = dst + (size_t(tile) * nb + b) * Q6K_TILE_BLOCK_BYTES;
  uint8_t* out = base + size_t(lane) * 16;
  // nibble words
  for (int s = 0; s < 8; ++s) {
    uint32_t w[4];
    for (int j = 0; j < 4; ++j) {
      uint32_t word = 0;
      for (int i = 0; i < 4; ++i) {
        const uint32_t a = q6_value(blk, q6_elem(s, j, i)) & 15;
        const uint32_t c = q6_value(blk, q6_elem(s + 8, j, i)) & 15;
        word |= (a | (c << 4)) << (8 * i);
      }
      w[j] = word;
    }
    *reinterpret_cast<uint4*>(out + size_t(s) * 16 * TILE) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  // high-bit words: h = 2s + jj -> chunk 8 + h/4, word h%4
  for (int c = 0; c < 4; ++c) {
    uint32_t w[4];
    for (int k = 0; k < 4; ++k) {
      const int h = 4 * c + k, s = h >> 1, jj = h & 1;
      uint32_t word = 0;
      for (int i = 0; i < 4; ++i) {
        const uint32_t b0 = q6_value(blk, q6_elem(s, 2 * jj, i)) >> 4;
        const uint32_t b1 = q6_value(blk, q6_elem(s, 2 * jj + 1, i)) >> 4;
        const uint32_t b2 = q6_value(blk, q6_elem(s + 8, 2 * jj, i)) >> 4;
        const uint32_t b3 = q6_value(blk, q6_elem(s + 8, 2 * jj + 1, i)) >> 4;
        word |= (b0 | (b1 << 2) | (b2 << 4) | (b3 << 6)) << (8 * i);
      }
      w[k] = word;
    }
    *reinterpret_cast<uint4*>(out + size_t(8 + c) * 16 * TILE) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  {
    uint32_t w[4];
    for (int k = 0; k < 4; ++k)
      w[k] = blk[192 + 4 * k] | (blk[193 + 4 * k] << 8) | (blk[194 + 4 * k] << 16) | (uint32_t(blk[195 + 4 * k]) << 24);
    *reinterpret_cast<uint4*>(out + size_t(12) * 16 * TILE) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  *reinterpret_cast<uint16_t*>(base + Q6K_DPLANE_OFFSET + size_t(lane) * 2) = uint16_t(blk[208] | (blk[209] << 8));
}

// ---- dequantize from the tile layout ------------------------------------------
//
// The per-row pieces below are shared by the dequantize kernels and by the
// dequantized matmul, so the bit-exact dequant test covers both.

// (q4k_dequant_chunk / q6k_dequant_group: hc_unpack.cuh)

__global__ void hc_dequant_q4k_kernel(const uint8_t* __restrict__ w, float* __restrict__ out, int rows, int nb) {
  const size_t t = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
  if (t >= size_t(rows) * nb) return;
  const int row = int(t / nb), b = int(t % nb);
  const uint8_t* tb = w + (size_t(row / TILE) * nb + b) * Q4K_TILE_BLOCK_BYTES;
  float* o = out + size_t(row) * nb * QK + size_t(b) * QK;
  for (int ch = 0; ch < 8; ++ch) q4k_dequant_chunk(tb, row % TILE, ch, o);
}

__global__ void hc_dequant_q6k_kernel(const uint8_t* __restrict__ w, float* __restrict__ out, int rows, int nb) {
  const size_t t = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
  if (t >= size_t(rows) * nb) return;
  const int row = int(t / nb), b = int(t % nb);
  const uint8_t* tb = w + (size_t(row / TILE) * nb + b) * Q6K_TILE_BLOCK_BYTES;
  float* o = out + size_t(row) * nb * QK + size_t(b) * QK;
  for (int s = 0; s < 8; ++s) q6k_dequant_group(tb, row % TILE, s, o);
}

// ---- dequantized matmul (hp_matmul_dequantized_f32, lib.rs:103-154) ---------
//
// out[col * rows + row] = the sequential f32 sum over k of
// fround(w[row][k] * x[col][k]), w the bit-exact dequantized row: one
// thread per (row, column) runs the reference's own chain
// sum = fround(sum + fround(w * x)) in index order (no fused multiply-add,
// no reassociation), so the result is the reference's bit for bit.
// CTA = one 32-row tile x NC columns: NC chain warps (lane = row) and eight
// dequant warps.  The tile's raw 256-blocks (and, for 16-byte aligned
// inputs, the columns' input slices) stream through a ring of DM_NS
// shared-memory slots, one bulk copy each issued DM_NS blocks ahead; per
// block the dequant warps turn a staged raw block into rows (row stride 260
// floats: 16-byte reads by lane = row hit distinct banks) in one half of a
// double buffer while the chain warps walk the other half, four elements per
// pair of 16-byte reads; one CTA barrier per block.  The chain's dependent
// adds are the bound.
constexpr int DM_DQ_WARPS = 8;
constexpr int DM_ROW = QK + 4;  // floats per staged row
constexpr int DM_NS = 4;        // raw ring slots
constexpr size_t DM_RAW = Q6K_TILE_BLOCK_BYTES;  // the larger raw block (16-byte multiple)

__host__ __device__ constexpr size_t dm_slot_bytes(int nc) { return DM_RAW + size_t(nc) * QK * 4; }

template <int NC>
__global__ void __launch_bounds__(32 * (NC + DM_DQ_WARPS)) hc_dequant_matmul_kernel(
    const uint8_t* __restrict__ w, int type, int nb, int rows, const float* __restrict__ x, int K, int cols,
    float* __restrict__ out, int x_bulk, int* err) {
  extern __shared__ __align__(16) float dm_smem[];  // ws [2][32][DM_ROW], xs [2][NC][256], raw ring [DM_NS][slot]
  __shared__ __align__(8) uint64_t full[DM_NS];
  float* ws = dm_smem;
  float* xs = dm_smem + 2 * TILE * DM_ROW;
  uint8_t* ring = reinterpret_cast<uint8_t*>(xs + 2 * NC * QK);
  const int tile = int(blockIdx.x), col0 = int(blockIdx.y) * NC;
  const int warp = int(threadIdx.x) >> 5, lane = int(threadIdx.x) & 31;
  const int ncols = min(NC, cols - col0);
  const uint32_t ub = uint32_t(type == TYPE_Q4_K ? Q4K_TILE_BLOCK_BYTES : Q6K_TILE_BLOCK_BYTES);
  const int dt = int(threadIdx.x) - 32 * NC;  // dequant thread index (< 0: a chain warp)
  int issued = 0;
  auto issue = [&](int b) {  // dequant thread 0: block b into its slot
    ++issued;
    const int sl = b % DM_NS;
    uint8_t* dst = ring + size_t(sl) * dm_slot_bytes(NC);
    mbar_expect_tx(&full[sl], ub + (x_bulk ? uint32_t(ncols) * QK * 4u : 0u));
    bulk_copy_g2s(dst, w + (size_t(tile) * nb + b) * ub, ub, &full[sl]);
    if (x_bulk)
      for (int c = 0; c < ncols; ++c)
        bulk_copy_g2s(dst + DM_RAW + size_t(c) * QK * 4, x + size_t(col0 + c) * K + size_t(b) * QK, QK * 4u,
                      &full[sl]);
  };
  bool ok = true;
  auto fill = [&](int b, int buf) {  // dequant warps: staged block b -> rows and inputs of half `buf`
    const int sl = b % DM_NS;
    const uint8_t* raw = ring + size_t(sl) * dm_slot_bytes(NC);
    if (ok && !mbar_wait_parity(&full[sl], uint32_t(b / DM_NS) & 1u, err)) ok = false;
    if (!ok) return;
    float* wb = ws + buf * TILE * DM_ROW;
    for (int task = dt; task < TILE * 8; task += 32 * DM_DQ_WARPS) {  // (row, 32-element part)
      const int r = task >> 3, part = task & 7;
      if (type == TYPE_Q4_K) q4k_dequant_chunk(raw, r, part, wb + r * DM_ROW);
      else q6k_dequant_group(raw, r, part, wb + r * DM_ROW);
    }
    float* xb = xs + buf * NC * QK;
    const float* xr = reinterpret_cast<const float*>(raw + DM_RAW);
    for (int i = dt; i < ncols * QK; i += 32 * DM_DQ_WARPS)
      xb[i] = x_bulk ? xr[i] : x[size_t(col0 + i / QK) * K + size_t(b) * QK + i % QK];
  };
  if (dt == 0) {
    for (int s = 0; s < DM_NS; ++s) mbar_init(&full[s], 1);
    for (int b = 0; b < nb && b < DM_NS; ++b) issue(b);
  }
  __syncthreads();
  if (dt >= 0) fill(0, 0);
  __syncthreads();
  if (dt == 0 && DM_NS < nb) issue(DM_NS);  // slot 0 is free again
  float sum = 0.0f;
  for (int b = 0; b < nb; ++b) {
    const int buf = b & 1;
    if (warp < NC) {
      if (warp < ncols) {
        const float4* wr = reinterpret_cast<const float4*>(ws + buf * TILE * DM_ROW + lane * DM_ROW);
        const float4* xc = reinterpret_cast<const float4*>(xs + (buf * NC + warp) * QK);
#pragma unroll 8
        for (int i = 0; i < QK / 4; ++i) {
          const float4 a = wr[i], v = xc[i];
          sum = __fadd_rn(sum, __fmul_rn(a.x, v.x));
          sum = __fadd_rn(sum, __fmul_rn(a.y, v.y));
          sum = __fadd_rn(sum, __fmul_rn(a.z, v.z));
          sum = __fadd_rn(sum, __fmul_rn(a.w, v.w));
        }
      }
    } else if (dt >= 0 && b + 1 < nb) {
      fill(b + 1, buf ^ 1);
    }
    __syncthreads();  // block b consumed, block b + 1 staged, its raw slot free
    if (dt == 0 && ok && b + 1 + DM_NS < nb) issue(b + 1 + DM_NS);
  }
  const int row = tile * TILE + lane;
  if (warp < ncols && row < rows) out[size_t(col0 + warp) * rows + row] = sum;
  if (dt == 0 && !ok)  // let the copies in flight land before the CTA exits
    for (int b = max(0, issued - DM_NS); b < issued; ++b)
      mbar_wait_parity(&full[b % DM_NS], uint32_t(b / DM_NS) & 1u, nullptr);
}

template <int NC>
static cudaError_t launch_dm(int type, const uint8_t* w, int nb, int rows, int rows_pad, const float* x, int K,
                             int cols, float* out, cudaStream_t stream) {
  constexpr size_t smem = sizeof(float) * (2 * TILE * DM_ROW + 2 * NC * QK) + DM_NS * dm_slot_bytes(NC);
  static std::atomic<uint64_t> attr{0};
  const cudaError_t ea = once_per_current_device(attr, [] {
    return cudaFuncSetAttribute(hc_dequant_matmul_kernel<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(smem));
  });
  if (ea != cudaSuccess) return ea;
  // the input slices go by bulk copy when every slice starts on 16 bytes
  const int x_bulk = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (size_t(K) * 4) % 16 == 0;
  const dim3 grid(unsigned(rows_pad / TILE), unsigned((cols + NC - 1) / NC));
  hc_dequant_matmul_kernel<NC><<<grid, 32 * (NC + DM_DQ_WARPS), smem, stream>>>(w, type, nb, rows, x, K, cols, out,
                                                                               x_bulk, device_status_word());
  return cudaGetLastError();
}

cudaError_t launch_dequant_matmul(int type, const uint8_t* w, int nb, int rows, int rows_pad, const float* x, int K,
                                  int cols, float* out, cudaStream_t stream) {
  if (cols <= 0 || rows <= 0) return cudaSuccess;
  if (cols == 1) return launch_dm<1>(type, w, nb, rows, rows_pad, x, K, cols, out, stream);
  if (cols == 2) return launch_dm<2>(type, w, nb, rows, rows_pad, x, K, cols, out, stream);
  if (cols <= 4) return launch_dm<4>(type, w, nb, rows, rows_pad, x, K, cols, out, stream);
  return launch_dm<8>(type, w, nb, rows, rows_pad, x, K, cols, out, stream);
}

cudaError_t launch_repack(int type, const uint8_t* src, uint8_t* dst, int rows, int rows_pad, int nb,
                          cudaStream_t stream) {
  const size_t n = size_t(rows_pad) * nb;
  const int threads = 128;
  const unsigned blocks = unsigned((n + threads - 1) / threads);
  if (type == TYPE_Q4_K) hc_repack_q4k_kernel<<<blocks, threads, 0, stream>>>(src, dst, rows, rows_pad, nb);
  else hc_repack_q6k_kernel<<<blocks, threads, 0, stream>>>(src, dst, rows, rows_pad, nb);
  return cudaGetLastError();
}

cudaError_t launch_dequant(int type, const uint8_t* w, float* out, int rows, int nb, cudaStream_t stream) {
  const size_t n = size_t(rows) * nb;
  const int threads = 128;
  const unsigned blocks = unsigned((n + threads - 1) / threads);
  if (type == TYPE_Q4_K) hc_dequant_q4k_kernel<<<blocks, threads, 0, stream>>>(w, out, rows, nb);
  else hc_dequant_q6k_kernel<<<blocks, threads, 0, stream>>>(w, out, rows, nb);
  return cudaGetLastError();
}

}  // namespace hc
