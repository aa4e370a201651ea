// hc_exact.cuh -- the K-quant x Q8_K row dot in the reference's own f32
// order, for one 32-row tile (lane = row).
//
// vec_dot_q4_k_q8_k_prepared (lib.rs:2117-2172) and
// vec_dot_q6_k_q8_k_prepared (lib.rs:1924-1968) keep eight f32 lane
// accumulators, lane = element index mod 8 (accumulate_scaled_i8_i8_32_lanes
// :2443-2501, ..._16_lanes :2265-2313), and per 256-block b add
//     sums[l] += (d_b * d8_b) * aux32_b[l]        (l = 0..7, f32, no FMA)
//     sumf    -= (dmin_b * d8_b) * sumi_b          (Q4_K only)
// in block order; the row result is sumf + (((0 + sums[0]) + sums[1]) ...
// + sums[7]) (Q6_K: the lane total alone).  The integer parts aux32_b[l] and
// sumi_b are exact; reproducing every f32 rounding in that order makes the
// GPU row dot equal the reference's bit for bit.
//
// Here the per-block integers come from the row-tile layout (hc_common.cuh):
//   Q4_K: word l of quant pair p holds lane l of groups 2p (low nibbles) and
//         2p + 1 (high nibbles); plane-A activation word l of group g holds
//         lane l of that group, so one dp4a per (pair, lane, half) is one
//         lane's 4-element partial of one 32-group;
//   Q6_K: nibble/high-bit word j of 16-group s holds elements
//         {16s+2j, 16s+2j+8} (lane 2j) in bytes 0-1 and {16s+2j+1, 16s+2j+9}
//         (lane 2j+1) in bytes 2-3, as does plane-B activation word j; the
//         6-bit values are made signed (q - 32) per byte and each lane's two
//         bytes are taken with a mask.
#pragma once
#include "hc_common.cuh"
#include "hc_unpack.cuh"

namespace hc {

// One column's exact per-block integers for one row.
struct BlockInts {
  int aux[8];  // aux32[l]
  int msum;    // Q4_K: sum_g mn_g * bsums32_g (sumi); Q6_K: unused
};

// Q4_K block of one row (unit chunk source `r`: chunk(0) = header, chunk(1..8)
// = quant words) against one plane-A record `rec`.
template <class Src>
__device__ __forceinline__ void q4k_lanes(const Src& r, const Q4KHeader& hd, const uint8_t* rec, BlockInts& o) {
#pragma unroll
  for (int l = 0; l < 8; ++l) o.aux[l] = 0;
#pragma unroll
  for (int pp = 0; pp < 4; ++pp) {
    const uint4 u0 = r.chunk(1 + 2 * pp), u1 = r.chunk(2 + 2 * pp);
    const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    const uint4 a0 = *reinterpret_cast<const uint4*>(rec + 64 * pp);
    const uint4 a1 = *reinterpret_cast<const uint4*>(rec + 64 * pp + 16);
    const uint4 a2 = *reinterpret_cast<const uint4*>(rec + 64 * pp + 32);
    const uint4 a3 = *reinterpret_cast<const uint4*>(rec + 64 * pp + 48);
    const uint32_t al[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const uint32_t ah[8] = {a2.x, a2.y, a2.z, a2.w, a3.x, a3.y, a3.z, a3.w};
    const int s0 = hd.sc(2 * pp), s1 = hd.sc(2 * pp + 1);
#pragma unroll
    for (int l = 0; l < 8; ++l) {
      o.aux[l] += s0 * dp4a(w[l] & 0x0f0f0f0fu, al[l], 0);
      o.aux[l] += s1 * dp4a((w[l] >> 4) & 0x0f0f0f0fu, ah[l], 0);
    }
  }
  const uint4 bs = *reinterpret_cast<const uint4*>(rec + Q8A_BS);
  int ms = __dp2a_lo(int(bs.x), int(hd.mn_lo), 0);
  ms = __dp2a_hi(int(bs.y), int(hd.mn_lo), ms);
  ms = __dp2a_lo(int(bs.z), int(hd.mn_hi), ms);
  o.msum = __dp2a_hi(int(bs.w), int(hd.mn_hi), ms);
}

// Q6_K block of one row against one plane-B record.
template <class Src>
__device__ __forceinline__ void q6k_lanes(const Src& r, const uint8_t* rec, BlockInts& o) {
  const uint4 scv = r.chunk(12);
  const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
#pragma unroll
  for (int l = 0; l < 8; ++l) o.aux[l] = 0;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const uint4 nv = r.chunk(s);
    const uint32_t nw[4] = {nv.x, nv.y, nv.z, nv.w};
    const uint4 hv = r.chunk(8 + (s >> 1));
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
    const int sa = int(int8_t((scw[s >> 2] >> (8 * (s & 3))) & 0xff));
    const int sb = int(int8_t((scw[(s + 8) >> 2] >> (8 * ((s + 8) & 3))) & 0xff));
    const uint4 A = *reinterpret_cast<const uint4*>(rec + 16 * s);
    const uint4 B = *reinterpret_cast<const uint4*>(rec + 16 * (s + 8));
    const uint32_t av[4] = {A.x, A.y, A.z, A.w}, bv[4] = {B.x, B.y, B.z, B.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t ua, ub;
      q6k_unpack(nw[j], hw[2 * (s & 1) + (j >> 1)], j & 1, ua, ub);
      // q - 32 per byte: every byte is 0..63, so no borrow crosses a byte
      const uint32_t qa = __vsub4(ua, 0x20202020u), qb = __vsub4(ub, 0x20202020u);
      o.aux[2 * j] += sa * dp4a(qa & 0x0000ffffu, av[j], 0) + sb * dp4a(qb & 0x0000ffffu, bv[j], 0);
      o.aux[2 * j + 1] += sa * dp4a(qa & 0xffff0000u, av[j], 0) + sb * dp4a(qb & 0xffff0000u, bv[j], 0);
    }
  }
  o.msum = 0;
}

// The eight lane accumulators and sumf of one (row, column), advanced block by
// block exactly as the reference does.
struct LaneChain {
  float s[8];
  float m;  // sumf
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int l = 0; l < 8; ++l) s[l] = 0.0f;
    m = 0.0f;
  }
  // d = f16(d_b) * d8_b, dm = f16(dmin_b) * d8_b (each rounded once, as the
  // prepared f32 scales times q8.d[block]); Q6_K passes has_min = false.
  __device__ __forceinline__ void add_block(const BlockInts& b, float d, float dm, bool has_min) {
#pragma unroll
    for (int l = 0; l < 8; ++l) s[l] = __fadd_rn(s[l], __fmul_rn(d, float(b.aux[l])));
    if (has_min) m = __fsub_rn(m, __fmul_rn(dm, float(b.msum)));
  }
  // sumf + sum of the lanes (lib.rs:2171); Q6_K: the lane sum (lib.rs:1967).
  __device__ __forceinline__ float total(bool has_min) const {
    float t = 0.0f;
#pragma unroll
    for (int l = 0; l < 8; ++l) t = __fadd_rn(t, s[l]);
    return has_min ? __fadd_rn(m, t) : t;
  }
};

}  // namespace hc
