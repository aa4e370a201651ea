// hc_prefetch.cu -- L2 prefetch of a decode layer's later weights.
//
// A decode step at batch 1 is a chain of dependent launches; while the
// attention of a layer runs (its sequential chains keep few SMs busy and HBM
// mostly idle), nothing reads the layer's output-projection and FFN weights
// yet.  This kernel, launched on a side stream that forks from the step
// after the QKV projection, walks those weights with
// cp.async.bulk.prefetch.L2 (no registers or shared memory consumed, no
// data returned) so that the GEMVs that follow find them in the 126 MB L2.
// It waits on nothing and nothing waits on it inside the layer: the side
// stream joins the step only at its end.
#include "hc_common.cuh"
#include "hc_kernels.cuh"

namespace hc {

namespace {

constexpr uint32_t PF_CHUNK = 32 * 1024;  // bytes per prefetch instruction

__global__ void __launch_bounds__(128) hc_l2_prefetch_kernel(const __grid_constant__ PrefetchList l) {
  size_t chunks[PREFETCH_MAX_RANGES];
  size_t total = 0;
#pragma unroll
  for (int i = 0; i < PREFETCH_MAX_RANGES; ++i) {
    chunks[i] = i < l.n ? (l.bytes[i] + PF_CHUNK - 1) / PF_CHUNK : 0;
    total += chunks[i];
  }
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  for (size_t c = size_t(blockIdx.x) * blockDim.x + threadIdx.x; c < total; c += stride) {
    size_t cc = c;
    int r = 0;
    while (r < l.n - 1 && cc >= chunks[r]) cc -= chunks[r++];
    const size_t off = cc * PF_CHUNK;
    const size_t left = l.bytes[r] - off;
    const uint32_t n = uint32_t(left < PF_CHUNK ? left : PF_CHUNK) & ~15u;
    if (n == 0) continue;
    const char* p = static_cast<const char*>(l.ptr[r]) + off;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(n) : "memory");
  }
}

}  // namespace

cudaError_t launch_l2_prefetch(const PrefetchList& l, cudaStream_t st) {
  if (l.n <= 0) return cudaSuccess;
  for (int i = 0; i < l.n; ++i)
    if ((reinterpret_cast<uintptr_t>(l.ptr[i]) & 15) != 0) return cudaErrorInvalidValue;
  hc_l2_prefetch_kernel<<<16, 128, 0, st>>>(l);
  return cudaGetLastError();
}

}  // namespace hc
