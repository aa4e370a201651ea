// hc_sample.cu -- the reference's token sampler on the device.
//
// Restates generation.ts:85-165 (token_sampling_distribution and
// sample_next_token) for one candidate list as the top-k entry points return
// it (value descending, then id ascending: the sampler's own sort order):
//   greedy            -> the first candidate, no draw;
//   top = the first max(1, top_k) candidates;
//   top-p nucleus     -> softmax of the values (f64 exp of value - max, a
//                        sequential f64 sum), the prefix whose mass first
//                        reaches top_p (the boundary candidate kept);
//   probabilities     -> softmax of value / temperature over the nucleus;
//   draw              -> the mulberry32-style generator of generation.ts:74-83
//                        advanced once from `state`, uniform in [0, 1);
//   inverse CDF       -> the first candidate whose running f64 sum exceeds the
//                        draw (the last one otherwise).
// The sums run in the reference's order; the exps are the device's f64 exp,
// which may differ from the host library's in the last bit, so a draw within
// ~1e-16 of a cumulative boundary could land on the neighbouring candidate.
// The chosen token's row of an f32 table [table_rows][hidden] times `scale`
// (f64 product rounded to f32) is written for the next draft step's input,
// so a chain of draft steps and draws runs without the host; a token outside
// the table (the empty id -1) leaves the row untouched.
#include <cmath>

#include "../../include/heliocuda.h"
#include "hc_common.cuh"
#include "hc_internal.h"

namespace hc {
namespace {

constexpr int SMP_MAX = 1024;  // candidates one launch samples (one thread each)

__device__ __forceinline__ uint32_t rng_draw(uint32_t state, double* u) {
  state += 0x6D2B79F5u;
  uint32_t v = state;
  v = (v ^ (v >> 15)) * (v | 1u);
  v ^= v + (v ^ (v >> 7)) * (v | 61u);
  *u = double(v ^ (v >> 14)) / 4294967296.0;
  return state;
}

__global__ void __launch_bounds__(SMP_MAX) hc_sample_kernel(const int32_t* __restrict__ ids,
                                                         const float* __restrict__ vals, int n, int top_k,
                                                         double top_p, double temperature, int greedy,
                                                         uint32_t state, int32_t* __restrict__ out_token,
                                                         const float* __restrict__ table, int table_rows, int hidden,
                                                         double scale, float* __restrict__ row_out) {
  __shared__ double e[SMP_MAX];
  __shared__ double s_mx;
  __shared__ int s_keep, s_token;
  const int t = int(threadIdx.x);
  const int m = max(1, min(n, top_k));  // the top-k survivors
  if (greedy) {
    if (t == 0) s_token = ids[0];
  } else {
    const double v = t < m ? double(vals[t]) : 0.0;
    // top-p: softmax of the values over the m survivors
    if (t == 0) {
      double mx = -INFINITY;
      for (int i = 0; i < m; ++i) mx = fmax(mx, double(vals[i]));
      s_mx = mx;
      s_keep = m;
    }
    __syncthreads();
    if (top_p < 1.0 && m > 1) {
      if (t < m) e[t] = exp(v - s_mx);
      __syncthreads();
      if (t == 0) {
        double s = 0.0;
        for (int i = 0; i < m; ++i) s += e[i];
        int keep = 1;
        if (s > 0.0 && isfinite(s)) {
          double cum = 0.0;
          keep = m;
          for (int i = 0; i < m; ++i) {
            cum += e[i] / s;
            if (cum >= top_p) {
              keep = i + 1;
              break;
            }
          }
        } else {
          // a degenerate softmax is one-hot on the first candidate, whose
          // mass 1 reaches any top_p
          keep = 1;
        }
        s_keep = keep;
      }
      __syncthreads();
    }
    const int keep = s_keep;
    // probabilities: softmax of value / temperature over the nucleus
    if (t == 0) {
      double mx = -INFINITY;
      for (int i = 0; i < keep; ++i) mx = fmax(mx, double(vals[i]) / temperature);
      s_mx = mx;
    }
    __syncthreads();
    if (t < keep) e[t] = exp(v / temperature - s_mx);
    __syncthreads();
    if (t == 0) {
      double s = 0.0;
      for (int i = 0; i < keep; ++i) s += e[i];
      const bool one_hot = !(s > 0.0 && isfinite(s));
      double u;
      rng_draw(state, &u);
      double cum = 0.0;
      int tok = ids[keep - 1];
      for (int i = 0; i < keep; ++i) {
        cum += one_hot ? (i == 0 ? 1.0 : 0.0) : e[i] / s;
        if (u < cum) {
          tok = ids[i];
          break;
        }
      }
      s_token = tok;
    }
  }
  __syncthreads();
  const int tok = s_token;
  if (t == 0) *out_token = tok;
  if (table != nullptr && tok >= 0 && tok < table_rows)  // ids outside the table are not read
    for (int i = t; i < hidden; i += int(blockDim.x))
      row_out[i] = float(double(table[size_t(tok) * size_t(hidden) + size_t(i)]) * scale);
}

}  // namespace
}  // namespace hc

extern "C" {

int hpc_sample_candidates(const int32_t* d_ids, const float* d_vals, size_t n, size_t top_k, double top_p,
                          double temperature, int greedy, uint32_t rng_state, int32_t* d_token, const float* d_table,
                          size_t table_rows, size_t hidden, double scale, float* d_row_out, void* stream) {
  if (n < 1 || n > size_t(hc::SMP_MAX) || top_k < 1) return hpc_fail(HPC_ERR_SHAPE, "sample: %zu candidates", n);
  if (!greedy && !(temperature > 0.0)) return hpc_fail(HPC_ERR_ARG, "sample: temperature %g", temperature);
  if (!d_ids || !d_vals || !d_token || (d_table && (!d_row_out || hidden == 0 || table_rows == 0)))
    return hpc_fail(HPC_ERR_ARG, "null pointer");
  if (table_rows > size_t(INT32_MAX) || hidden > size_t(INT32_MAX)) return hpc_fail(HPC_ERR_SHAPE, "sample: table");
  const int threads = greedy ? 256 : hc::SMP_MAX;
  hc::hc_sample_kernel<<<1, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      d_ids, d_vals, int(n), int(top_k > n ? n : top_k), top_p, temperature, greedy, rng_state, d_token, d_table,
      int(table_rows), int(hidden), scale, d_row_out);
  HPC_CK(cudaGetLastError(), "sample launch");
  return HPC_OK;
}

}  // extern "C"
