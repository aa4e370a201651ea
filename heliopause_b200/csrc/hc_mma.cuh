// hc_mma.cuh -- Q4_K / Q6_K x Q8_K block products on the tensor cores
// (mma.sync s8 x s8 -> s32), shared by the wide matmul (hc_gemm_tc.cu) and
// the narrow 3..8-column GEMV (hc_gemv_mma.cu).
//
// Same arithmetic as the dp4a GEMV (hc_gemv_body.cuh, i.e.
// vec_dot_q4_k_q8_k / vec_dot_q6_k_q8_k, lib.rs:2117-2172 / 1924-1968): the
// integer sum of every (row, column, sub-block) is exact, then scaled by the
// sub-block's integer scale, summed over the block in int32, and combined
// with d, dmin and the activation's d in f32 once per 256-block.
//
// The row-tile layout already stores the 4-bit / 6-bit values in the order
// the dp4a path pairs them with the record bytes; read with lane = (row,
// 4-word group), the same words are exactly the A fragments of m16n8k32
// (Q4_K) / m16n8k16 (Q6_K), and the record words are the B fragments, so no
// repack is needed.
#pragma once
#include <cuda_fp16.h>

#include "hc_common.cuh"
#include "hc_unpack.cuh"

namespace hc {

// f16 bits -> f32 by the hardware conversion: exact for every finite value
// (subnormals included) and the infinities, so equal to float16_to_float32
// (lib.rs:2507-2532) except for NaN payloads.  One instruction instead of the
// bit-assembly of f16_bits_to_f32; the block products decode four headers per
// lane per block, where it matters.
__device__ __forceinline__ float f16_to_f32_hw(uint32_t bits) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
}

__device__ __forceinline__ Q4KHeader q4k_header_hw(const uint4 h) {
  Q4KHeader r;
  r.d = f16_to_f32_hw(h.x & 0xffffu);
  r.dmin = f16_to_f32_hw(h.x >> 16);
  r.sc_lo = h.y & 0x3f3f3f3fu;
  r.mn_lo = h.z & 0x3f3f3f3fu;
  r.sc_hi = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
  r.mn_hi = ((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u);
  return r;
}

__device__ __forceinline__ void mma_k32(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// Unsigned A (0..255) x signed B.
__device__ __forceinline__ void mma_k32_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void mma_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
               : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
               : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// One 256-block of a warp's 32 rows x 8 NG columns.  `unit` is the tile's
// block in the row-tile layout (hc_common.cuh), `act` the Q8_K record of
// column 0 for this block (plane A for Q4_K, B for Q6_K), column c's record at
// act + c * cs.  Lane (g = lane / 4, t = lane % 4): rows 16 mg + g and
// 16 mg + g + 8, columns 8 ng + 2t, + 1 (the m16n8 accumulator layout).
template <int TYPE, int NG>
__device__ __forceinline__ void tc_block(const uint8_t* unit, const uint8_t* act, int cs, float (&acc)[2][NG][4],
                                         int g, int t) {
  int isum[2][NG][4];
#pragma unroll
  for (int mg = 0; mg < 2; ++mg)
#pragma unroll
    for (int ng = 0; ng < NG; ++ng)
#pragma unroll
      for (int r = 0; r < 4; ++r) isum[mg][ng][r] = 0;
  if constexpr (TYPE == TYPE_Q4_K) {
    // One column group (the narrow GEMV): the high nibbles are used in place
    // (w & 0xf0f0f0f0 = 16 q) as unsigned A, which saves a shift per word;
    // their sums are 16x and kept apart, then divided exactly by 16 (every
    // term is a multiple of 16; |sum| < 4 * 63 * 32 * 240 * 128 < 2^31).
    constexpr bool HI16 = NG == 1;
    int ihi[2][NG][4];
#pragma unroll
    for (int mg = 0; mg < 2; ++mg)
#pragma unroll
      for (int ng = 0; ng < NG; ++ng)
#pragma unroll
        for (int r = 0; r < 4; ++r) ihi[mg][ng][r] = 0;
    Q4KHeader hd[2][2];
#pragma unroll
    for (int mg = 0; mg < 2; ++mg)
#pragma unroll
      for (int h = 0; h < 2; ++h)
        hd[mg][h] = q4k_header_hw(*reinterpret_cast<const uint4*>(unit + (16 * mg + 8 * h + g) * 16));
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      uint32_t w[2][4];  // [mg][row g low word, row g+8 low word, row g high word, row g+8 high word]
#pragma unroll
      for (int mg = 0; mg < 2; ++mg) {
        w[mg][0] = lds32(unit + (1 + 2 * pp) * 512 + (16 * mg + g) * 16 + 4 * t);
        w[mg][1] = lds32(unit + (1 + 2 * pp) * 512 + (16 * mg + g + 8) * 16 + 4 * t);
        w[mg][2] = lds32(unit + (2 + 2 * pp) * 512 + (16 * mg + g) * 16 + 4 * t);
        w[mg][3] = lds32(unit + (2 + 2 * pp) * 512 + (16 * mg + g + 8) * 16 + 4 * t);
      }
#pragma unroll
      for (int ng = 0; ng < NG; ++ng) {
        const uint8_t* rec = act + (8 * ng + g) * cs + 64 * pp + 4 * t;
        const uint32_t bl0 = lds32(rec), bl1 = lds32(rec + 16), bh0 = lds32(rec + 32), bh1 = lds32(rec + 48);
#pragma unroll
        for (int mg = 0; mg < 2; ++mg) {
          int clo[4], chi[4];
          mma_k32(clo, w[mg][0] & 0x0f0f0f0fu, w[mg][1] & 0x0f0f0f0fu, w[mg][2] & 0x0f0f0f0fu,
                  w[mg][3] & 0x0f0f0f0fu, bl0, bl1);
          if constexpr (HI16) {
            mma_k32_u8s8(chi, w[mg][0] & 0xf0f0f0f0u, w[mg][1] & 0xf0f0f0f0u, w[mg][2] & 0xf0f0f0f0u,
                         w[mg][3] & 0xf0f0f0f0u, bh0, bh1);
          } else {
            mma_k32(chi, (w[mg][0] >> 4) & 0x0f0f0f0fu, (w[mg][1] >> 4) & 0x0f0f0f0fu,
                    (w[mg][2] >> 4) & 0x0f0f0f0fu, (w[mg][3] >> 4) & 0x0f0f0f0fu, bh0, bh1);
          }
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const Q4KHeader& h = hd[mg][r >> 1];
            if constexpr (HI16) {
              isum[mg][ng][r] += h.sc(2 * pp) * clo[r];
              ihi[mg][ng][r] += h.sc(2 * pp + 1) * chi[r];
            } else {
              isum[mg][ng][r] += h.sc(2 * pp) * clo[r] + h.sc(2 * pp + 1) * chi[r];
            }
          }
        }
      }
    }
    if constexpr (HI16) {
#pragma unroll
      for (int mg = 0; mg < 2; ++mg)
#pragma unroll
        for (int ng = 0; ng < NG; ++ng)
#pragma unroll
          for (int r = 0; r < 4; ++r) isum[mg][ng][r] += ihi[mg][ng][r] >> 4;
    }
#pragma unroll
    for (int ng = 0; ng < NG; ++ng) {
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const uint8_t* rec = act + (8 * ng + 2 * t + cc) * cs;
        const uint4 bs = *reinterpret_cast<const uint4*>(rec + Q8A_BS);
        const float d8 = *reinterpret_cast<const float*>(rec + Q8A_D);
#pragma unroll
        for (int mg = 0; mg < 2; ++mg)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const Q4KHeader& hh = hd[mg][h];
            int ms = __dp2a_lo(int(bs.x), int(hh.mn_lo), 0);
            ms = __dp2a_hi(int(bs.y), int(hh.mn_lo), ms);
            ms = __dp2a_lo(int(bs.z), int(hh.mn_hi), ms);
            ms = __dp2a_hi(int(bs.w), int(hh.mn_hi), ms);
            const int r = 2 * h + cc;
            acc[mg][ng][r] += __fmul_rn(hh.d, d8) * float(isum[mg][ng][r]) - __fmul_rn(hh.dmin, d8) * float(ms);
          }
      }
    }
  } else {
    uint32_t scw[2][2][4];
    float dw[2][2];
#pragma unroll
    for (int mg = 0; mg < 2; ++mg)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = 16 * mg + 8 * h + g;
        const uint4 s4 = *reinterpret_cast<const uint4*>(unit + 12 * 512 + row * 16);
        scw[mg][h][0] = s4.x;
        scw[mg][h][1] = s4.y;
        scw[mg][h][2] = s4.z;
        scw[mg][h][3] = s4.w;
        dw[mg][h] = f16_to_f32_hw(reinterpret_cast<const uint16_t*>(unit + Q6K_DPLANE_OFFSET)[row]);
      }
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      uint32_t ua[2][2], ub[2][2];  // [mg][row g, row g+8]
#pragma unroll
      for (int mg = 0; mg < 2; ++mg)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = 16 * mg + 8 * h + g;
          const uint32_t nw = lds32(unit + s * 512 + row * 16 + 4 * t);
          const uint32_t hw = lds32(unit + (8 + (s >> 1)) * 512 + row * 16 + 4 * (2 * (s & 1) + (t >> 1)));
          q6k_unpack(nw, hw, t & 1, ua[mg][h], ub[mg][h]);
        }
#pragma unroll
      for (int ng = 0; ng < NG; ++ng) {
        const uint8_t* rec = act + (8 * ng + g) * cs + 4 * t;
        const uint32_t ba = lds32(rec + 16 * s), bb = lds32(rec + 16 * (s + 8));
#pragma unroll
        for (int mg = 0; mg < 2; ++mg) {
          int ca[4], cb[4];
          mma_k16(ca, ua[mg][0], ua[mg][1], ba);
          mma_k16(cb, ub[mg][0], ub[mg][1], bb);
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const uint32_t* sw = scw[mg][r >> 1];
            const int sa = int(int8_t((sw[s >> 2] >> (8 * (s & 3))) & 0xff));
            const int sb = int(int8_t((sw[(s + 8) >> 2] >> (8 * ((s + 8) & 3))) & 0xff));
            isum[mg][ng][r] += sa * ca[r] + sb * cb[r];
          }
        }
      }
    }
#pragma unroll
    for (int ng = 0; ng < NG; ++ng) {
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const uint8_t* rec = act + (8 * ng + 2 * t + cc) * cs;
        const uint4 b0 = *reinterpret_cast<const uint4*>(rec + Q8B_BS);
        const uint4 b1 = *reinterpret_cast<const uint4*>(rec + Q8B_BS + 16);
        const float d8 = *reinterpret_cast<const float*>(rec + Q8B_D);
#pragma unroll
        for (int mg = 0; mg < 2; ++mg)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t* sw = scw[mg][h];
            int corr = __dp2a_lo(int(b0.x), int(sw[0]), 0);
            corr = __dp2a_hi(int(b0.y), int(sw[0]), corr);
            corr = __dp2a_lo(int(b0.z), int(sw[1]), corr);
            corr = __dp2a_hi(int(b0.w), int(sw[1]), corr);
            corr = __dp2a_lo(int(b1.x), int(sw[2]), corr);
            corr = __dp2a_hi(int(b1.y), int(sw[2]), corr);
            corr = __dp2a_lo(int(b1.z), int(sw[3]), corr);
            corr = __dp2a_hi(int(b1.w), int(sw[3]), corr);
            const int r = 2 * h + cc;
            acc[mg][ng][r] += __fmul_rn(dw[mg][h], d8) * float(isum[mg][ng][r] - 32 * corr);
          }
      }
    }
  }
}

}  // namespace hc
