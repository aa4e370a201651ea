// hc_decmath.cuh -- device arithmetic of the decoder layer math shared by the
// decode-step kernels (hc_decode.cu, hc_attx.cu): programmatic-dependent-launch
// controls, the two f16 codecs of the reference, f64 reductions, the
// per-head QK-norm + RoPE and the GEGLU activation.  Every
// rounding point follows packages/engine/src/runner/wasm/layers.ts and
// packages/engine/wasm-kernels/src/lib.rs as cited per function.
#pragma once
#include <cmath>

#include <cuda_fp16.h>

#include "hc_common.cuh"

namespace hc {

__device__ __forceinline__ void pdl_trigger() {
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.launch_dependents;");
#endif
}
__device__ __forceinline__ void pdl_wait() {
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}

// Eight consecutive floats (16-byte aligned) into registers.
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// ---- f16 codecs ---------------------------------------------------------------

// quant.ts:632-669 float32ToFloat16 (the TS codec used by layers.ts): round
// to nearest even, |x| >= 65504 clamps to 65504, |x| < 2^-24 flushes to zero.
__device__ __forceinline__ float round_f16_ts(float x) {
  const float a = fabsf(x);
  if (x != x) return x;
  if (a >= 65504.0f) return a == INFINITY ? x : copysignf(65504.0f, x);
  if (a < 5.9604644775390625e-8f) return copysignf(0.0f, x);
  return __half2float(__float2half_rn(x));
}

// lib.rs:2534-2568 float32_to_float16 (the Rust codec used for the attention
// query, lib.rs:590-597): the dropped bits round half UP, overflow clamps to
// 0x7bff, NaN -> 0x7e00.  Returns the f16 value widened back to f32.
__device__ __forceinline__ float round_f16_rust(float v) {
  // Branch-free on the f32 bits (one result per case, then a select):
  //   f16 normal range: add half an f16 ulp (bit 12) and clear the 13 bits
  //     f16 drops -- a carry moves into the exponent as the codec's does --
  //     then clamp anything that reached 2^16 to 65504 (0x7bff);
  //   f16 subnormal range (f32 exponents 102..112): round the 24-bit
  //     significand half up at 2^-24, scaled back exactly;
  //   below: signed zero; Inf keeps its sign; NaN becomes 0x7e00.
  const uint32_t bits = __float_as_uint(v), sign = bits & 0x80000000u, a = bits & 0x7fffffffu;
  const int exp = int(a >> 23);
  uint32_t rn = (a + 0x1000u) & 0xffffe000u;
  rn = rn >= 0x47800000u ? 0x477fe000u : rn;
  const int shift = min(max(126 - exp, 1), 31);
  const uint32_t m = (a & 0x7fffffu) | 0x800000u;
  const uint32_t hs = (m + (1u << (shift - 1))) >> shift;
  const uint32_t fs = __float_as_uint(float(hs) * 5.9604644775390625e-8f);
  const uint32_t r = exp >= 113 ? rn : (exp >= 102 ? fs : 0u);
  if (exp == 255) return (a & 0x7fffffu) ? __uint_as_float(0x7fc00000u) : __uint_as_float(sign | 0x7f800000u);
  return __uint_as_float(sign | r);
}

// ---- block reductions -----------------------------------------------------------

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Sum over a CTA of `warps` warps (all threads call it).
__device__ __forceinline__ double block_sum_d(double v, double* scratch, int warps) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < warps; ++w) t += scratch[w];
  return t;
}

// One warp: QK-norm (f64 sum of squares, layers.ts:871-885 normHeads) of a
// 256-vector held 8 values per lane (lane L: dimensions 8L..8L+7), optional
// weight w (preloaded, same layout), optional NeoX RoPE (layers.ts:990-1033;
// pair (i, i+128) sits in lanes L and L+16) with the lane's eight cos/sin
// entries c8/s8 (pair indices (L mod 16)*8 .. +7); products rounded to f32
// as in the reference.
__device__ __forceinline__ void head_norm_rope(float (&x)[8], const float (&w)[8], bool has_w, bool rope,
                                               const double (&c8)[8], const double (&s8)[8], double eps, int lane) {
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += double(x[i]) * double(x[i]);
  ss = warp_sum_d(ss);
  const double sc = 1.0 / sqrt(ss / 256.0 + eps);
  if (!has_w) {
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = float(double(x[i]) * sc);
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = float((double(x[i]) * sc) * double(w[i]));
  if (!rope) return;
  float partner[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, x[i], 16);
  const bool first = lane < 16;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const double x0 = first ? x[i] : partner[i];
    const double x1 = first ? partner[i] : x[i];
    x[i] = first ? float(x0 * c8[i]) - float(x1 * s8[i]) : float(x0 * s8[i]) + float(x1 * c8[i]);
  }
}

// The lane's eight cos and sin entries of one token's row of the RoPE tables.
__device__ __forceinline__ void load_rope8(const double* cos_row, const double* sin_row, int lane, double (&c8)[8],
                                           double (&s8)[8]) {
  const double2* c = reinterpret_cast<const double2*>(cos_row + (lane & 15) * 8);
  const double2* sn = reinterpret_cast<const double2*>(sin_row + (lane & 15) * 8);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const double2 a = c[i], b = sn[i];
    c8[2 * i] = a.x;
    c8[2 * i + 1] = a.y;
    s8[2 * i] = b.x;
    s8[2 * i + 1] = b.y;
  }
}

// layers.ts:1062-1076 gelu (tanh form) with the TS f16 codec on input and
// output; |x| >= 10 short-circuits.
__device__ __forceinline__ double gelu_ts(float v) {
  if (v <= -10.0f) return 0.0;
  if (v >= 10.0f) return double(v);
  const double x = double(round_f16_ts(v));
  const float xx = float(x * x);
  const float poly = float(1.0 + double(float(0.044715 * double(xx))));
  const float lin = float(0.7978845608028654 * x);  // Math.sqrt(2 / Math.PI) as a double
  const float inner = float(double(lin) * double(poly));
  const float hlf = float(0.5 * x);
  const float act = float(double(hlf) * double(float(1.0 + tanh(double(inner)))));
  return double(round_f16_ts(act));
}

}  // namespace hc
