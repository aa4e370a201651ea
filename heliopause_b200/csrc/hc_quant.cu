// hc_quant.cu -- Q8_K activation quantization on the GPU, bit-exact to
// quantize_q8_k (packages/engine/wasm-kernels/src/lib.rs:1774-1811).
//
// One warp per (column, 256-element block); lane L owns elements 8L..8L+7.
// The block amax is a warp reduction over (|x|, index) pairs that keeps the
// larger |x| and, on equal |x|, the LOWER index -- the same element the
// reference's sequential "first strictly greater" scan keeps.  Then
// inv = -127/max (IEEE division), q = min(127, roundf(inv*x)) saturated to
// int8, d = 1/inv, all with explicit round-to-nearest intrinsics so no
// multiply-add contraction can change a bit.
#include <climits>

#include "hc_common.cuh"
#include "hc_kernels.cuh"

namespace hc {

__device__ __forceinline__ int8_t sat_i8(float v) {
  // Rust `as i8`: NaN -> 0, saturate, truncate toward zero (v is integral).
  if (v != v) return 0;
  v = fmaxf(v, -128.0f);
  return static_cast<int8_t>(__float2int_rz(v));
}

__device__ __forceinline__ uint32_t byte_at(const uint8_t* s, int i) { return s[i]; }

template <bool NATURAL>
__global__ void __launch_bounds__(256) q8k_quantize_kernel(const float* __restrict__ x, int K, int cols, Q8Buf q,
                                                           int8_t* __restrict__ nat_qs,
                                                           int16_t* __restrict__ nat_bs32,
                                                           float* __restrict__ nat_d) {
  __shared__ __align__(16) uint8_t stage[8][256];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int nb = K / QK;
  const int gw = blockIdx.x * 8 + wib;
  if (gw >= nb * cols) return;
  const int col = gw / nb, b = gw % nb;
  const size_t base = size_t(col) * K + size_t(b) * QK;
  uint8_t* recA = q.a + (size_t(col) * nb + b) * Q8A_REC;
  uint8_t* recB = q.b + (size_t(col) * nb + b) * Q8B_REC;
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif

  const float4* src = reinterpret_cast<const float4*>(x + base + lane * 8);
  float4 v0 = __ldg(src), v1 = __ldg(src + 1);
  float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};

  float amax = 0.0f, val = 0.0f;
  int idx = INT_MAX;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float a = fabsf(v[i]);
    if (a > amax) {
      amax = a;
      val = v[i];
      idx = lane * 8 + i;
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    float oa = __shfl_xor_sync(0xffffffffu, amax, off);
    int oi = __shfl_xor_sync(0xffffffffu, idx, off);
    float ov = __shfl_xor_sync(0xffffffffu, val, off);
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
      int8_t qi = sat_i8(fminf(roundf(__fmul_rn(inv, v[i])), 127.0f));
      s8 += qi;
      uint32_t u = uint32_t(uint8_t(qi));
      if (i < 4) w0 |= u << (8 * i);
      else w1 |= u << (8 * (i - 4));
    }
    d = __fdiv_rn(1.0f, inv);
  }
  *reinterpret_cast<uint2*>(&stage[wib][lane * 8]) = make_uint2(w0, w1);
  __syncwarp();

  // Permuted copies (see hc_common.cuh): lane L writes words 2L and 2L+1.
  const uint8_t* st = stage[wib];
  uint32_t p32[2], p16[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int W = 2 * lane + k;
    {
      const int g = W >> 3, l = W & 7, o = 32 * g + l;
      p32[k] = byte_at(st, o) | (byte_at(st, o + 8) << 8) | (byte_at(st, o + 16) << 16) | (byte_at(st, o + 24) << 24);
    }
    {
      const int s = W >> 2, j = W & 3, o = 16 * s + 2 * j;
      p16[k] = byte_at(st, o) | (byte_at(st, o + 8) << 8) | (byte_at(st, o + 1) << 16) | (byte_at(st, o + 9) << 24);
    }
  }
  *reinterpret_cast<uint2*>(recA + lane * 8) = make_uint2(p32[0], p32[1]);
  *reinterpret_cast<uint2*>(recB + lane * 8) = make_uint2(p16[0], p16[1]);

  // 16-element sums: lanes 2s, 2s+1.  32-element sums: lanes 4g..4g+3.
  int s16 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);
  int s32 = s16 + __shfl_xor_sync(0xffffffffu, s16, 2);
  if ((lane & 1) == 0) reinterpret_cast<int16_t*>(recB + Q8B_BS)[lane >> 1] = int16_t(s16);
  if ((lane & 3) == 0) reinterpret_cast<int16_t*>(recA + Q8A_BS)[lane >> 2] = int16_t(s32);
  if (lane == 0) {
    *reinterpret_cast<float*>(recA + Q8A_D) = d;
    *reinterpret_cast<float*>(recB + Q8B_D) = d;
  }
  if (NATURAL) {
    *reinterpret_cast<uint2*>(nat_qs + base + lane * 8) = make_uint2(w0, w1);
    if ((lane & 3) == 0) nat_bs32[size_t(col) * (K / 32) + b * 8 + (lane >> 2)] = int16_t(s32);
    if (lane == 0) nat_d[size_t(col) * nb + b] = d;
  }
}

cudaError_t launch_q8k_quantize(const float* x, int K, int cols, const Q8Buf& q, int8_t* nat_qs, int16_t* nat_bs32,
                                float* nat_d, cudaStream_t stream) {
  const int warps = (K / QK) * cols;
  const unsigned blocks = unsigned((warps + 7) / 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (nat_qs) return cudaLaunchKernelEx(&cfg, q8k_quantize_kernel<true>, x, K, cols, q, nat_qs, nat_bs32, nat_d);
  return cudaLaunchKernelEx(&cfg, q8k_quantize_kernel<false>, x, K, cols, q, (int8_t*)nullptr, (int16_t*)nullptr,
                            (float*)nullptr);
}

}  // namespace hc
