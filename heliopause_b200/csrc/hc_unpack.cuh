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

}  // namespace hc
