// hc_unpack.cuh -- register-level unpack helpers shared by the dequantize,
// GEMV and LM-head kernels, so the bit-exact dequant test also covers the
// unpack arithmetic the matmuls use.
#pragma once
#include "hc_common.cuh"

namespace hc {

// Q4_K block header (first 16 bytes): d, dmin (f16) and the 12 packed scale
// bytes.  The 6-bit scales/mins of get_scale_min_k4 (lib.rs:2250-2259) are
// produced four at a time as packed bytes:
//   j < 4 : sc = q[j] & 63,                     mn = q[j+4] & 63
//   j >= 4: sc = (q[j+4] & 15) | (q[j-4] >> 6) << 4,
//           mn = (q[j+4] >> 4) | (q[j]   >> 6) << 4
struct Q4KHeader {
  float d, dmin;
  uint32_t sc_lo, sc_hi, mn_lo, mn_hi;  // bytes: sc0..3, sc4..7, mn0..3, mn4..7
  __device__ __forceinline__ int sc(int g) const {
    return int(((g < 4 ? sc_lo : sc_hi) >> (8 * (g & 3))) & 0xff);
  }
  __device__ __forceinline__ int mn(int g) const {
    return int(((g < 4 ? mn_lo : mn_hi) >> (8 * (g & 3))) & 0xff);
  }
};

__device__ __forceinline__ Q4KHeader q4k_header(const uint4 h) {
  Q4KHeader r;
  r.d = f16_bits_to_f32(h.x & 0xffffu);
  r.dmin = f16_bits_to_f32(h.x >> 16);
  r.sc_lo = h.y & 0x3f3f3f3fu;
  r.mn_lo = h.z & 0x3f3f3f3fu;
  r.sc_hi = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
  r.mn_hi = ((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u);
  return r;
}

// Q6_K: rebuild the unsigned 6-bit values (0..63) of one nibble word.
// `odd` = j & 1 selects which 2-bit field pair of the high-bit word applies.
// ua = group s (low nibbles), ub = group s+8 (high nibbles).
__device__ __forceinline__ void q6k_unpack(uint32_t nw, uint32_t hw, int odd, uint32_t& ua, uint32_t& ub) {
  const int sh = odd ? 2 : 0;
  ua = (nw & 0x0f0f0f0fu) | ((hw << (4 - sh)) & 0x30303030u);
  ub = ((nw >> 4) & 0x0f0f0f0fu) | ((hw >> sh) & 0x30303030u);
}

// Streaming 16-byte load that does not allocate in L1 (weights are read once
// per launch; L1 is kept for the activation words every lane broadcasts).
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint32_t ld_stream_u16(const uint16_t* p) {
  unsigned short r;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}

// ---- dequantize one row of a tile-block -------------------------------------
// Shared by the dequantize kernels, the dequantized matmul and the draft
// head's gathered rows, so the bit-exact dequant test covers all of them.

// Row `r` of a Q4_K tile-block: the 32 values of quant chunk ch (0..7) into
// o[0..256): elements 64p + j (low nibbles) and 64p + 32 + j (high), p = ch/2.
__device__ __forceinline__ void q4k_dequant_chunk(const uint8_t* tb, int r, int ch, float* o) {
  const uint4* c = reinterpret_cast<const uint4*>(tb) + r;
  const Q4KHeader hd = q4k_header(c[0]);
  const uint4 v = c[size_t(1 + ch) * TILE];
  const uint32_t words[4] = {v.x, v.y, v.z, v.w};
  const int p = ch >> 1;
  const float d1 = __fmul_rn(hd.d, float(hd.sc(2 * p))), d2 = __fmul_rn(hd.d, float(hd.sc(2 * p + 1)));
  const float m1 = __fmul_rn(hd.dmin, float(hd.mn(2 * p))), m2 = __fmul_rn(hd.dmin, float(hd.mn(2 * p + 1)));
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int l = 4 * (ch & 1) + k;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t byte = (words[k] >> (8 * i)) & 0xff;
      const int j = l + 8 * i;  // position inside the 32-byte pair
      o[64 * p + j] = __fsub_rn(__fmul_rn(d1, float(byte & 15)), m1);
      o[64 * p + 32 + j] = __fsub_rn(__fmul_rn(d2, float(byte >> 4)), m2);
    }
  }
}

// Row `r` of a Q6_K tile-block: the 32 values of 16-groups s and s + 8
// (s = 0..7) into o[0..256).
__device__ __forceinline__ void q6k_dequant_group(const uint8_t* tb, int r, int s, float* o) {
  const uint4* c = reinterpret_cast<const uint4*>(tb) + r;
  const float d = f16_bits_to_f32(reinterpret_cast<const uint16_t*>(tb + Q6K_DPLANE_OFFSET)[r]);
  const uint4 scv = c[12 * TILE];
  const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
  const uint4 nv = c[size_t(s) * TILE];
  const uint32_t nw[4] = {nv.x, nv.y, nv.z, nv.w};
  const uint4 hv = c[size_t(8 + (s >> 1)) * TILE];
  const uint32_t hw4[4] = {hv.x, hv.y, hv.z, hv.w};
  const int sa = int(int8_t((scw[s >> 2] >> (8 * (s & 3))) & 0xff));
  const int sb = int(int8_t((scw[(s + 8) >> 2] >> (8 * ((s + 8) & 3))) & 0xff));
  const float da = __fmul_rn(d, float(sa)), db = __fmul_rn(d, float(sb));
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t hw = hw4[2 * (s & 1) + (j >> 1)];
    uint32_t ua, ub;
    q6k_unpack(nw[j], hw, j & 1, ua, ub);
    const int off[4] = {0, 8, 1, 9};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int qa = int((ua >> (8 * i)) & 0xff) - 32;
      const int qb = int((ub >> (8 * i)) & 0xff) - 32;
      o[16 * s + 2 * j + off[i]] = __fmul_rn(da, float(qa));
      o[16 * (s + 8) + 2 * j + off[i]] = __fmul_rn(db, float(qb));
    }
  }
}

// One thread per (row, block).
}  // namespace hc
