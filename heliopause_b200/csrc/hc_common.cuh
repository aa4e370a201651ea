// hc_common.cuh -- shared definitions for the heliocuda kernels (sm_100a).
//
// HBM layouts
// -----------
// Weights are uploaded in GGUF block layout and repacked once into "row tiles":
// 32 consecutive output rows form a tile, and each 16-byte chunk of a block is
// stored for all 32 rows side by side, so one warp-wide 16-byte load fetches
// that chunk for 32 rows as one contiguous 512-byte segment.  Each thread of a
// warp owns one row: no cross-lane reduction is needed inside a block.  Rows
// past row_count are zero-filled (d = 0), so a tile is always complete.
//
//   Q4_K (144 B/block/row):  9 chunks per (tile, block)
//     chunk 0      : the original 16-byte header  d | dmin | 12 scale bytes
//     chunk 1 + c  : quant bytes, permuted per 32-byte pair p = c/2:
//                    word l (l = 0..7) of pair p = bytes {l, l+8, l+16, l+24}
//                    of that pair, so word l's low nibbles are lane l of group
//                    2p and its high nibbles lane l of group 2p+1 (lane = index
//                    mod 8, the accumulator lane of lib.rs:2443-2466).
//   Q6_K (210 B/block/row):  13 chunks + a 2-byte d plane per (tile, block)
//     chunks 0..7  : nibble words NW[s][j] (s = 0..7, j = 0..3): byte i holds
//                    the low 4 bits of element e_i(s,j) (low nibble) and of
//                    e_i(s+8,j) (high nibble), with e(s,j) = 16s + {2j, 2j+8,
//                    2j+1, 2j+9}
//     chunks 8..11 : high-bit words HW[s][jj] (16 words): byte i bits 0-1,
//                    2-3, 4-5, 6-7 = top 2 bits of e_i(s,2jj), e_i(s,2jj+1),
//                    e_i(s+8,2jj), e_i(s+8,2jj+1)
//     chunk 12     : the 16 int8 sub-block scales, original order
//     d plane      : 32 x f16 after the chunks
//
// Q8_K activations ("q8 buffer") are written by the quantize kernels as two
// block-interleaved planes, one record per (column, 256-block), so a CTA can
// stage the slice it needs with one bulk copy per column:
//   plane A (Q4_K consumers), 288 B/record:
//     [0,256)   p32: per 32-group g, word l = q{32g+l, +8, +16, +24}
//     [256,272) eight int16 32-element sums   [272,276) d (f32)
//   plane B (Q6_K consumers), 304 B/record:
//     [0,256)   p16: per 16-group s, word j = q{16s+2j, 16s+2j+8, 16s+2j+1, 16s+2j+9}
//     [256,288) sixteen int16 16-element sums [288,292) d (f32)
// Record of (col, block b) sits at plane + (col * nb + b) * record_bytes.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "hc_once.h"

namespace hc {

// once_per_device (hc_once.h) on the calling thread's current device: a
// launcher's one-time kernel-attribute set-up, done again on each device.
template <class F>
inline cudaError_t once_per_current_device(std::atomic<uint64_t>& done, F&& set) {
  int dev = 0;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  return once_per_device<cudaError_t>(done, dev, static_cast<F&&>(set));
}

constexpr int QK = 256;
constexpr int TILE = 32;
constexpr int TYPE_Q4_K = 1;
constexpr int TYPE_Q6_K = 3;

constexpr int Q4K_CHUNKS = 9;
constexpr int Q6K_CHUNKS = 13;
constexpr size_t Q4K_TILE_BLOCK_BYTES = 144 * TILE;  // 4608
constexpr size_t Q6K_TILE_BLOCK_BYTES = 210 * TILE;  // 6720
constexpr size_t Q6K_DPLANE_OFFSET = Q6K_CHUNKS * 16 * TILE;  // 6656

__host__ __device__ inline size_t tile_block_bytes(int type) {
  return type == TYPE_Q4_K ? Q4K_TILE_BLOCK_BYTES : Q6K_TILE_BLOCK_BYTES;
}

constexpr int Q8A_REC = 288;
constexpr int Q8B_REC = 304;
constexpr int Q8A_BS = 256, Q8A_D = 272;
constexpr int Q8B_BS = 256, Q8B_D = 288;

struct Q8Buf {
  uint8_t* a;  // plane A
  uint8_t* b;  // plane B
  int K;
  int cols;
};

__host__ __device__ inline int q8_rec_bytes(int type) { return type == TYPE_Q4_K ? Q8A_REC : Q8B_REC; }

// Bytes needed for `cols` columns of width K (both planes, 256-byte aligned).
inline size_t q8buf_bytes(int K, int cols) {
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t recs = size_t(cols) * (K / 256);
  return al(recs * Q8A_REC) + al(recs * Q8B_REC);
}

inline Q8Buf q8buf_carve(void* base, int K, int cols) {
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t recs = size_t(cols) * (K / 256);
  Q8Buf q;
  q.a = static_cast<uint8_t*>(base);
  q.b = q.a + al(recs * Q8A_REC);
  q.K = K;
  q.cols = cols;
  return q;
}

// Exact f16 -> f32 on the bit pattern, identical to float16_to_float32
// (lib.rs:2507-2532) for every input including subnormals and NaN payloads.
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
  uint32_t sign = (h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t f = h & 0x3ffu;
  uint32_t bits;
  if (e == 0) {
    if (f == 0) {
      bits = sign;
    } else {
      int shift = __clz(f) - 21;  // moves the leading 1 to bit 10
      f = (f << shift) & 0x3ffu;
      bits = sign | (uint32_t(-14 - shift + 127) << 23) | (f << 13);
    }
  } else if (e == 31) {
    bits = sign | 0x7f800000u | (f << 13);
  } else {
    bits = sign | ((e + 112u) << 23) | (f << 13);
  }
  return __uint_as_float(bits);
}

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
  return __dp4a(int(a), int(b), c);
}

}  // namespace hc
