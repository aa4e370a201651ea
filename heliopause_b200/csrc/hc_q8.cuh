// hc_q8.cuh -- warp-level Q8_K quantization of one 256-element block,
// bit-exact to quantize_q8_k (packages/engine/wasm-kernels/src/lib.rs:1774-1811),
// writing the plane-A / plane-B records of hc_common.cuh.  Shared by the
// standalone quantize kernel and the decode-step epilogues (norms, attention
// combine, GEGLU) that produce the next matmul's input directly.
#pragma once
#include <climits>

#include "hc_common.cuh"

namespace hc {

__device__ __forceinline__ int8_t q8_sat_i8(float v) {
  // Rust `as i8`: NaN -> 0, saturate, truncate toward zero (v is integral).
  if (v != v) return 0;
  v = fmaxf(v, -128.0f);
  return static_cast<int8_t>(__float2int_rz(v));
}

// Quantizes the 256 values v[0..7] of lanes 0..31 (lane L holds elements
// 8L..8L+7 of the block) into recA/recB.  `stage` is 256 bytes of this
// warp's shared memory.  Optionally returns the natural-order words and d.
__device__ __forceinline__ void q8k_block_warp(const float (&v)[8], int lane, uint8_t* stage, uint8_t* recA,
                                               uint8_t* recB, uint32_t* nat_w0 = nullptr, uint32_t* nat_w1 = nullptr,
                                               int* s32_out = nullptr, float* d_out = nullptr) {
  (void)stage;  // the byte transposes below run in registers
  float amax = 0.0f, val = 0.0f;
  int idx = INT_MAX;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = fabsf(v[i]);
    if (a > amax) {
      amax = a;
      val = v[i];
      idx = lane * 8 + i;
    }
  }
  // warp argmax of |v| with the lowest index on ties, as one 64-bit key:
  // amax >= 0, so its bits order like its value; the low word orders the
  // index in reverse
  unsigned long long key = (static_cast<unsigned long long>(__float_as_uint(amax)) << 32) | (0xffffffffu - unsigned(idx));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, key, off);
    key = o > key ? o : key;
  }
  amax = __uint_as_float(unsigned(key >> 32));
  idx = int(0xffffffffu - unsigned(key));
  val = __shfl_sync(0xffffffffu, val, (idx >> 3) & 31);  // the lane holding the argmax owns it as its `val`
  uint32_t w0 = 0, w1 = 0;
  int s8 = 0;
  float d = 0.0f;
  if (amax != 0.0f) {
    const float inv = __fdiv_rn(-127.0f, val);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int8_t qi = q8_sat_i8(fminf(roundf(__fmul_rn(inv, v[i])), 127.0f));
      s8 += qi;
      const uint32_t u = uint32_t(uint8_t(qi));
      if (i < 4) w0 |= u << (8 * i);
      else w1 |= u << (8 * (i - 4));
    }
    d = __fdiv_rn(1.0f, inv);
  }
  // Element e sits in lane e / 8, byte e % 8 of (w0, w1).  Both record
  // layouts gather bytes from the lane's own quad of lanes:
  //   plane A, word k of lane 4a+b: byte 2b+k of lanes 4a .. 4a+3;
  //   plane B, word k of lane 2c+e: bytes 4e+2k and 4e+2k+1 of lanes 2c, 2c+1.
  const int qb = lane & ~3;
  uint32_t a0[4], a1[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    a0[j] = __shfl_sync(0xffffffffu, w0, qb | j);
    a1[j] = __shfl_sync(0xffffffffu, w1, qb | j);
  }
  const int b = lane & 3;
  const uint32_t sel_ab = (b & 1) ? 0x7632u : 0x5410u;  // the two bytes 2(b&1), 2(b&1)+1 of both words
  const uint32_t x01 = __byte_perm(b < 2 ? a0[0] : a1[0], b < 2 ? a0[1] : a1[1], sel_ab);
  const uint32_t x23 = __byte_perm(b < 2 ? a0[2] : a1[2], b < 2 ? a0[3] : a1[3], sel_ab);
  const uint32_t p32_0 = __byte_perm(x01, x23, 0x6420u);
  const uint32_t p32_1 = __byte_perm(x01, x23, 0x7531u);
  const bool odd = (lane & 1) != 0, upper = (lane & 2) != 0;
  const uint32_t u0 = odd ? (upper ? a1[2] : a1[0]) : (upper ? a0[2] : a0[0]);
  const uint32_t u1 = odd ? (upper ? a1[3] : a1[1]) : (upper ? a0[3] : a0[1]);
  const uint32_t p16_0 = __byte_perm(u0, u1, 0x5140u);
  const uint32_t p16_1 = __byte_perm(u0, u1, 0x7362u);
  *reinterpret_cast<uint2*>(recA + lane * 8) = make_uint2(p32_0, p32_1);
  *reinterpret_cast<uint2*>(recB + lane * 8) = make_uint2(p16_0, p16_1);
  const int s16 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);
  const int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 2);
  if ((lane & 1) == 0) reinterpret_cast<int16_t*>(recB + Q8B_BS)[lane >> 1] = int16_t(s16);
  if ((lane & 3) == 0) reinterpret_cast<int16_t*>(recA + Q8A_BS)[lane >> 2] = int16_t(s32);
  if (lane == 0) {
    *reinterpret_cast<float*>(recA + Q8A_D) = d;
    *reinterpret_cast<float*>(recB + Q8B_D) = d;
  }
  if (nat_w0) {
    *nat_w0 = w0;
    *nat_w1 = w1;
    *s32_out = s32;
    *d_out = d;
  }
}

__device__ __forceinline__ uint8_t* q8_rec_a(const Q8Buf& q, int col, int b) {
  return q.a + (size_t(col) * (q.K / QK) + b) * Q8A_REC;
}
__device__ __forceinline__ uint8_t* q8_rec_b(const Q8Buf& q, int col, int b) {
  return q.b + (size_t(col) * (q.K / QK) + b) * Q8B_REC;
}

}  // namespace hc
