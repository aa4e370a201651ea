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
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float oa = __shfl_xor_sync(0xffffffffu, amax, off);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
    const float ov = __shfl_xor_sync(0xffffffffu, val, off);
    if (oa > amax || (oa == amax && oi < idx)) {
      amax = oa;
      idx = oi;
      val = ov;
    }
  }
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
  *reinterpret_cast<uint2*>(stage + lane * 8) = make_uint2(w0, w1);
  __syncwarp();
  uint32_t p32[2], p16[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int W = 2 * lane + k;
    {
      const int g = W >> 3, l = W & 7, o = 32 * g + l;
      p32[k] = uint32_t(stage[o]) | (uint32_t(stage[o + 8]) << 8) | (uint32_t(stage[o + 16]) << 16) |
               (uint32_t(stage[o + 24]) << 24);
    }
    {
      const int s = W >> 2, j = W & 3, o = 16 * s + 2 * j;
      p16[k] = uint32_t(stage[o]) | (uint32_t(stage[o + 8]) << 8) | (uint32_t(stage[o + 1]) << 16) |
               (uint32_t(stage[o + 9]) << 24);
    }
  }
  __syncwarp();
  *reinterpret_cast<uint2*>(recA + lane * 8) = make_uint2(p32[0], p32[1]);
  *reinterpret_cast<uint2*>(recB + lane * 8) = make_uint2(p16[0], p16[1]);
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
