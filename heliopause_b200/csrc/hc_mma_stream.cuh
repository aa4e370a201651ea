// hc_mma_stream.cuh -- the weight stream of the tensor-core GEMV and LM head
// (hc_gemv_mma.cu, hc_lmhead_mma.cu): every warp streams its items' units
// (one 256-block of one 32-row tile, contiguous in the row-tile layout)
// through its own ring of shared-memory slots, one cp.async.bulk per unit
// completing on the slot's mbarrier, and computes each with the tensor-core
// block products of hc_mma.cuh over an 8-column activation slice.
#pragma once
#include "hc_bulk.cuh"
#include "hc_common.cuh"
#include "hc_gemv_body.cuh"
#include "hc_kernels.cuh"
#include "hc_mma.cuh"

namespace hc {

constexpr int GM_COLS = 8;

// Column stride of an activation slice of nblk records per column: 16 bytes
// of padding put the eight columns' B-fragment words in distinct banks.
__host__ __device__ inline int gm_col_stride(int nblk, int rec) { return nblk * rec + 16; }

__host__ __device__ inline size_t gm_act_bytes(const GemvParams& p, int nblk) {
  bool a, b;
  gemv_planes(p, &a, &b);
  const size_t s = size_t(GM_COLS) * ((a ? gm_col_stride(nblk, Q8A_REC) : 0) + (b ? gm_col_stride(nblk, Q8B_REC) : 0));
  return (s + 15) / 16 * 16;
}

// Ring slot size: the largest unit among the launch's weights.
__host__ __device__ inline int gm_slot_bytes(const GemvParams& p) {
  bool a, b;
  gemv_planes(p, &a, &b);
  return unit_bytes(b ? TYPE_Q6_K : TYPE_Q4_K);
}

// Thread 0: the activation slice of columns col0 .. col0 + 7 (columns past
// ncols repeat the last real one, so the B fragments are always defined),
// blocks [kb0, kb0 + nblk), one bulk copy per column and plane, completing
// on `bar`.  The caller syncs the CTA before anyone waits on `bar`.
__device__ __forceinline__ void stage_act_slice8(const GemvParams& p, uint8_t* act_a, uint8_t* act_b, int cs_a,
                                                 int cs_b, int kb0, int nblk, uint64_t* bar) {
  if (threadIdx.x != 0) return;
  const uint32_t per_col = uint32_t(nblk) * uint32_t((act_a ? Q8A_REC : 0) + (act_b ? Q8B_REC : 0));
  mbar_init(bar, 1);
  mbar_expect_tx(bar, per_col * GM_COLS);
  for (int c = 0; c < GM_COLS; ++c) {
    const size_t rec0 = size_t(p.col0 + (c < p.ncols ? c : p.ncols - 1)) * p.nb + kb0;
    if (act_a) bulk_copy_g2s(act_a + size_t(c) * cs_a, p.q.a + rec0 * Q8A_REC, uint32_t(nblk * Q8A_REC), bar);
    if (act_b) bulk_copy_g2s(act_b + size_t(c) * cs_b, p.q.b + rec0 * Q8B_REC, uint32_t(nblk * Q8B_REC), bar);
  }
}

// One warp's unit stream: unit u is block u % bps of item item0 + (u / bps)
// * istride.  The units of an item are contiguous, so an item is its first
// unit's address and its type.
struct MmaStream {
  const GemvParams& p;
  int item0, istride, n, R, slot, lane, issued;
  uint8_t* ring;
  uint64_t* bars;
  const uint8_t* iss_base;  // lane 0's issue cursor: first unit of item iss_k
  int iss_type, iss_k;

  __device__ MmaStream(const GemvParams& p_, int item0_, int istride_, int nitems, uint8_t* ring_, int slot_,
                       uint64_t* bars_, int lane_)
      : p(p_), item0(item0_), istride(istride_), R(p_.ring), slot(slot_), lane(lane_), ring(ring_), bars(bars_) {
    n = item0 < nitems ? ((nitems - 1 - item0) / istride + 1) * p.bps : 0;
    issued = n < R ? n : R;
    iss_k = 0;
    iss_base = unit_addr(p, item0 < nitems ? item0 : 0, 0, &iss_type);
  }

  __device__ __forceinline__ void issue(int u) {  // lane 0, in increasing u
    const int k = u / p.bps;
    if (k != iss_k) {
      iss_k = k;
      iss_base = unit_addr(p, item0 + k * istride, 0, &iss_type);
    }
    const uint32_t ub = uint32_t(unit_bytes(iss_type));
    uint64_t* b = bars + (u % R);
    mbar_expect_tx(b, ub);
    bulk_copy_g2s(ring + size_t(u % R) * slot, iss_base + size_t(u % p.bps) * ub, ub, b);
  }

  // Before griddepcontrol.wait (the weights do not depend on the previous
  // kernel): lane 0 initializes the ring's barriers and fills it.
  __device__ __forceinline__ void prime() {
    if (lane == 0) {
      for (int s = 0; s < R; ++s) mbar_init(bars + s, 1);
      for (int u = 0; u < issued; ++u) issue(u);
    }
    __syncwarp();
  }

  // Streams every unit; `flush(item, acc)` receives each finished item's
  // 32 x 8 sums in the m16n8 accumulator layout (lane (g, t): rows
  // 16 mg + g + 8 (r >> 1), column 2 t + (r & 1)).  The activation slice
  // holds blocks [kb0, kb0 + nblk) of the launch's K range.  Returns false
  // after a bounded wait timed out; the copies still in flight have
  // then been waited for (bounded), so the CTA may exit.
  template <class Flush>
  __device__ __forceinline__ bool run(const uint8_t* act_a, const uint8_t* act_b, int cs_a, int cs_b, int kb0,
                                      bool ok, int g, int t, Flush& flush) {
    float acc[2][1][4];
#pragma unroll
    for (int mg = 0; mg < 2; ++mg)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[mg][0][r] = 0.0f;
    int u = 0, item = item0, j = 0, ty;
    unit_addr(p, item0, 0, &ty);
    for (; ok && u < n; ++u) {
      if (!mbar_wait_parity_sleep(bars + (u % R), uint32_t(u / R) & 1u, p.err)) {
        ok = false;
        break;
      }
      const uint8_t* unit = ring + size_t(u % R) * slot;
      const int jj = (item & (p.split - 1)) * p.bps + j - kb0;  // block inside the CTA's slice
      if (ty == TYPE_Q4_K) tc_block<TYPE_Q4_K, 1>(unit, act_a + jj * Q8A_REC, cs_a, acc, g, t);
      else tc_block<TYPE_Q6_K, 1>(unit, act_b + jj * Q8B_REC, cs_b, acc, g, t);
      __syncwarp();  // every lane has consumed the slot: refill it
      if (u + R < n) {
        if (lane == 0) issue(u + R);
        ++issued;
      }
      if (j == p.bps - 1) {
        flush(item, acc);
#pragma unroll
        for (int mg = 0; mg < 2; ++mg)
#pragma unroll
          for (int r = 0; r < 4; ++r) acc[mg][0][r] = 0.0f;
        item += istride;
        j = 0;
        if (u + 1 < n) unit_addr(p, item, 0, &ty);
      } else {
        ++j;
      }
    }
    if (!ok)
      for (; u < issued; ++u) mbar_wait_parity(bars + (u % R), uint32_t(u / R) & 1u, nullptr);
    return ok;
  }
};

}  // namespace hc
