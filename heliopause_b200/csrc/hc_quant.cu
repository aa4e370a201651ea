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
#include "hc_common.cuh"
#include "hc_kernels.cuh"
#include "hc_q8.cuh"

namespace hc {

template <bool NATURAL>
__global__ void __launch_bounds__(256) hc_q8k_quantize_kernel(const float* __restrict__ x, int K, int cols, Q8Buf q,
                                                           int8_t* __restrict__ nat_qs,
                                                           int16_t* __restrict__ nat_bs32,
                                                           float* __restrict__ nat_d) {
  __shared__ __align__(16) uint8_t stage[8][256];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int nb = K / QK;
  const int gw = blockIdx.x * 8 + wib;
#if __CUDA_ARCH__ >= 900
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
  if (gw >= nb * cols) return;
  const int col = gw / nb, b = gw % nb;
  const size_t base = size_t(col) * K + size_t(b) * QK;
  const float4* src = reinterpret_cast<const float4*>(x + base + lane * 8);
  const float4 v0 = __ldg(src), v1 = __ldg(src + 1);
  const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  uint32_t w0, w1;
  int s32;
  float d;
  q8k_block_warp(v, lane, stage[wib], q8_rec_a(q, col, b), q8_rec_b(q, col, b), &w0, &w1, &s32, &d);
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
  if (nat_qs) return cudaLaunchKernelEx(&cfg, hc_q8k_quantize_kernel<true>, x, K, cols, q, nat_qs, nat_bs32, nat_d);
  return cudaLaunchKernelEx(&cfg, hc_q8k_quantize_kernel<false>, x, K, cols, q, (int8_t*)nullptr, (int16_t*)nullptr,
                            (float*)nullptr);
}

}  // namespace hc
