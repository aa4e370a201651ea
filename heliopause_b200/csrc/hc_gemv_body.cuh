// hc_gemv_body.cuh -- the streaming core shared by the GEMV and LM-head
// kernels: per-block Q4_K / Q6_K x Q8_K dot products for one 32-row tile
// (lane = row) computed from registers, and the register double buffer that
// keeps two units (one 256-element block of one tile each) in flight per warp.
//
// Block math follows vec_dot_q4_k_q8_k_prepared (lib.rs:2117-2172) and
// vec_dot_q6_k_q8_k_prepared (lib.rs:1924-1968): exact int32 block sums
//   Q4_K: sum_g sc[g] * dot(q4, q8)_g  and  sum_g mn[g] * bsum32[g]
//   Q6_K: sum_s sc[s] * dot(q6 - 32, q8)_s
// combined per block as (d*d8)*isum - (dmin*d8)*msum in f32.
//
// Work decomposition (see hc_gemv.cu): an "item" is (tile, K part); the K
// range of a tile is split into p.split parts, item i = (i / split, i % split).
// A warp walks its items and streams their units through the double buffer,
// so the loads of the next unit (possibly of the next item) are in flight
// while the current one is computed.
#pragma once
#include "hc_bulk.cuh"
#include "hc_common.cuh"
#include "hc_exact.cuh"
#include "hc_kernels.cuh"
#include "hc_unpack.cuh"

namespace hc {

constexpr int UNIT_CHUNKS = Q6K_CHUNKS;  // register buffer sized for the larger type

// Activation records staged in shared memory (hc_common.cuh planes): record of
// (local column c, local block j) at act + (c*nblk + j)*rec.
struct ActSlice {
  const uint8_t* a;  // plane A records (Q4_K)
  const uint8_t* b;  // plane B records (Q6_K)
  int nblk;          // blocks per column in the slice
  int kb0;           // first block of the slice
};

// One unit in registers: UC = Q6K_CHUNKS holds either type; UC = Q4K_CHUNKS
// (launches whose weights are all Q4_K) holds Q4_K only and needs ~40 fewer
// registers per buffer.
template <int UC>
struct UnitRegsN {
  uint4 c[UC];
  uint32_t d;  // Q6_K d bits
};
using UnitRegs = UnitRegsN<UNIT_CHUNKS>;

// Streaming loads: evict-first, no L1 allocation (weights are read once).
template <int UC>
__device__ __forceinline__ void load_unit(UnitRegsN<UC>& r, const uint8_t* unit, int type, int lane) {
  const uint4* p = reinterpret_cast<const uint4*>(unit) + lane;
  if (UC == Q4K_CHUNKS || type == TYPE_Q4_K) {
#pragma unroll
    for (int k = 0; k < Q4K_CHUNKS; ++k) r.c[k] = __ldcs(p + k * TILE);
  } else {
#pragma unroll
    for (int k = 0; k < (UC > Q4K_CHUNKS ? Q6K_CHUNKS : 0); ++k) r.c[k] = __ldcs(p + k * TILE);
    r.d = __ldcs(reinterpret_cast<const unsigned short*>(unit + Q6K_DPLANE_OFFSET) + lane);
  }
}

// Where a unit's 16-byte chunks come from: a register buffer, or shared
// memory read chunk by chunk as the dot product consumes them.
template <int UC>
struct RegSrc {
  const UnitRegsN<UC>& r;
  __device__ __forceinline__ uint4 chunk(int k) const { return r.c[k]; }
  __device__ __forceinline__ uint32_t dbits() const { return r.d; }
};
struct SmemSrc {
  const uint4* p;       // the unit's first chunk for this lane (row)
  const uint16_t* dp;   // this lane's Q6_K d
  __device__ __forceinline__ uint4 chunk(int k) const { return p[k * TILE]; }
  __device__ __forceinline__ uint32_t dbits() const { return *dp; }
};

template <int NC, class Src>
__device__ __forceinline__ void q4k_src(const Src& r, int j, int ncols, const ActSlice& act, float (&acc)[NC]) {
  const Q4KHeader hd = q4k_header(r.chunk(0));
  int isum[NC];
#pragma unroll
  for (int col = 0; col < NC; ++col) isum[col] = 0;
#pragma unroll
  for (int pp = 0; pp < 4; ++pp) {
    const uint4 u0 = r.chunk(1 + 2 * pp), u1 = r.chunk(2 + 2 * pp);
    const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    const int s0 = hd.sc(2 * pp), s1 = hd.sc(2 * pp + 1);
#pragma unroll
    for (int col = 0; col < NC; ++col) {
      if (col < ncols) {
        const uint8_t* rec = act.a + (col * act.nblk + j) * Q8A_REC + 64 * pp;
        const uint4 a0 = *reinterpret_cast<const uint4*>(rec), a1 = *reinterpret_cast<const uint4*>(rec + 16);
        const uint4 a2 = *reinterpret_cast<const uint4*>(rec + 32), a3 = *reinterpret_cast<const uint4*>(rec + 48);
        const uint32_t al[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const uint32_t ah[8] = {a2.x, a2.y, a2.z, a2.w, a3.x, a3.y, a3.z, a3.w};
        int tl = 0, th = 0;
#pragma unroll
        for (int l = 0; l < 8; ++l) {
          tl = dp4a(w[l] & 0x0f0f0f0fu, al[l], tl);
          th = dp4a((w[l] >> 4) & 0x0f0f0f0fu, ah[l], th);
        }
        isum[col] += s0 * tl + s1 * th;
      }
    }
  }
#pragma unroll
  for (int col = 0; col < NC; ++col) {
    if (col < ncols) {
      const uint8_t* rec = act.a + (col * act.nblk + j) * Q8A_REC;
      const uint4 bs = *reinterpret_cast<const uint4*>(rec + Q8A_BS);
      int ms = __dp2a_lo(int(bs.x), int(hd.mn_lo), 0);
      ms = __dp2a_hi(int(bs.y), int(hd.mn_lo), ms);
      ms = __dp2a_lo(int(bs.z), int(hd.mn_hi), ms);
      ms = __dp2a_hi(int(bs.w), int(hd.mn_hi), ms);
      const float d8 = *reinterpret_cast<const float*>(rec + Q8A_D);
      acc[col] += __fmul_rn(hd.d, d8) * float(isum[col]) - __fmul_rn(hd.dmin, d8) * float(ms);
    }
  }
}

template <int NC, class Src>
__device__ __forceinline__ void q6k_src(const Src& r, int j, int ncols, const ActSlice& act, float (&acc)[NC]) {
  const float dw = f16_bits_to_f32(r.dbits());
  const uint4 scv = r.chunk(12);
  const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
  int isum[NC];
#pragma unroll
  for (int col = 0; col < NC; ++col) isum[col] = 0;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const uint4 nv = r.chunk(s);
    const uint32_t nw[4] = {nv.x, nv.y, nv.z, nv.w};
    const uint4 hv = r.chunk(8 + (s >> 1));
    const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
    uint32_t ua[4], ub[4];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) q6k_unpack(nw[jj], hw[2 * (s & 1) + (jj >> 1)], jj & 1, ua[jj], ub[jj]);
    const int sa = int(int8_t((scw[s >> 2] >> (8 * (s & 3))) & 0xff));
    const int sb = int(int8_t((scw[(s + 8) >> 2] >> (8 * ((s + 8) & 3))) & 0xff));
#pragma unroll
    for (int col = 0; col < NC; ++col) {
      if (col < ncols) {
        const uint8_t* rec = act.b + (col * act.nblk + j) * Q8B_REC;
        const uint4 A = *reinterpret_cast<const uint4*>(rec + 16 * s);
        const uint4 B = *reinterpret_cast<const uint4*>(rec + 16 * (s + 8));
        int ta = dp4a(ua[0], A.x, 0);
        ta = dp4a(ua[1], A.y, ta);
        ta = dp4a(ua[2], A.z, ta);
        ta = dp4a(ua[3], A.w, ta);
        int tb = dp4a(ub[0], B.x, 0);
        tb = dp4a(ub[1], B.y, tb);
        tb = dp4a(ub[2], B.z, tb);
        tb = dp4a(ub[3], B.w, tb);
        isum[col] += sa * ta + sb * tb;
      }
    }
  }
#pragma unroll
  for (int col = 0; col < NC; ++col) {
    if (col < ncols) {
      // The 6-bit values were used unsigned (0..63); subtract 32 * sum(sc * bsum16).
      const uint8_t* rec = act.b + (col * act.nblk + j) * Q8B_REC;
      const uint4 b0 = *reinterpret_cast<const uint4*>(rec + Q8B_BS);
      const uint4 b1 = *reinterpret_cast<const uint4*>(rec + Q8B_BS + 16);
      int corr = __dp2a_lo(int(b0.x), int(scw[0]), 0);
      corr = __dp2a_hi(int(b0.y), int(scw[0]), corr);
      corr = __dp2a_lo(int(b0.z), int(scw[1]), corr);
      corr = __dp2a_hi(int(b0.w), int(scw[1]), corr);
      corr = __dp2a_lo(int(b1.x), int(scw[2]), corr);
      corr = __dp2a_hi(int(b1.y), int(scw[2]), corr);
      corr = __dp2a_lo(int(b1.z), int(scw[3]), corr);
      corr = __dp2a_hi(int(b1.w), int(scw[3]), corr);
      const float d8 = *reinterpret_cast<const float*>(rec + Q8B_D);
      acc[col] += __fmul_rn(dw, d8) * float(isum[col] - 32 * corr);
    }
  }
}

// Loads one unit that was staged in shared memory into registers.
template <int UC>
__device__ __forceinline__ void load_unit_smem(UnitRegsN<UC>& r, const uint8_t* unit, int type, int lane) {
  const uint4* p = reinterpret_cast<const uint4*>(unit) + lane;
  if (UC == Q4K_CHUNKS || type == TYPE_Q4_K) {
#pragma unroll
    for (int k = 0; k < Q4K_CHUNKS; ++k) r.c[k] = p[k * TILE];
  } else {
#pragma unroll
    for (int k = 0; k < (UC > Q4K_CHUNKS ? Q6K_CHUNKS : 0); ++k) r.c[k] = p[k * TILE];
    r.d = reinterpret_cast<const uint16_t*>(unit + Q6K_DPLANE_OFFSET)[lane];
  }
}

template <int NC, int UC>
__device__ __forceinline__ void unit_compute(const UnitRegsN<UC>& r, int type, int j, int ncols, const ActSlice& act,
                                             float (&acc)[NC]) {
  const RegSrc<UC> src{r};
  if constexpr (UC == Q4K_CHUNKS) {
    q4k_src<NC>(src, j, ncols, act, acc);
  } else {
    if (type == TYPE_Q4_K) q4k_src<NC>(src, j, ncols, act, acc);
    else q6k_src<NC>(src, j, ncols, act, acc);
  }
}

// unit_compute in the reference's exact f32 order (hc_exact.cuh): the unit's
// per-lane integer sums of every column advance that column's eight lane
// accumulators (and sumf) by one block.
template <int NC, int UC>
__device__ __forceinline__ void unit_compute_exact(const UnitRegsN<UC>& r, int type, int j, int ncols,
                                                   const ActSlice& act, LaneChain (&acc)[NC]) {
  const RegSrc<UC> src{r};
  if (UC == Q4K_CHUNKS || type == TYPE_Q4_K) {
    const Q4KHeader hd = q4k_header(src.chunk(0));
#pragma unroll
    for (int col = 0; col < NC; ++col) {
      if (col < ncols) {
        const uint8_t* rec = act.a + (col * act.nblk + j) * Q8A_REC;
        BlockInts b;
        q4k_lanes(src, hd, rec, b);
        const float d8 = *reinterpret_cast<const float*>(rec + Q8A_D);
        acc[col].add_block(b, __fmul_rn(hd.d, d8), __fmul_rn(hd.dmin, d8), true);
      }
    }
  } else {
    const float dw = f16_bits_to_f32(src.dbits());
#pragma unroll
    for (int col = 0; col < NC; ++col) {
      if (col < ncols) {
        const uint8_t* rec = act.b + (col * act.nblk + j) * Q8B_REC;
        BlockInts b;
        q6k_lanes(src, rec, b);
        acc[col].add_block(b, __fmul_rn(dw, *reinterpret_cast<const float*>(rec + Q8B_D)), 0.0f, false);
      }
    }
  }
}

// unit_compute on a unit staged in shared memory, read chunk by chunk as the
// dot products consume it (no register buffer).
template <int NC, int UC>
__device__ __forceinline__ void unit_compute_smem(const uint8_t* unit, int type, int j, int ncols,
                                                  const ActSlice& act, float (&acc)[NC], int lane) {
  const SmemSrc src{reinterpret_cast<const uint4*>(unit) + lane,
                    reinterpret_cast<const uint16_t*>(unit + Q6K_DPLANE_OFFSET) + lane};
  if constexpr (UC == Q4K_CHUNKS) {
    q4k_src<NC>(src, j, ncols, act, acc);
  } else {
    if (type == TYPE_Q4_K) q4k_src<NC>(src, j, ncols, act, acc);
    else q6k_src<NC>(src, j, ncols, act, acc);
  }
}

__device__ __forceinline__ int seg_of(const GemvParams& p, int tile_g) {
  int si = 0;
#pragma unroll
  for (int i = 1; i < GEMV_MAXSEG; ++i)
    if (i < p.nseg && tile_g >= p.seg[i].tile_begin) si = i;
  return si;
}

// Position of one unit in a warp's stream.
struct UnitPos {
  int item;  // global item index
  int j;     // block offset inside the item's K part
};

// Address and type of unit j of an item.
__device__ __forceinline__ const uint8_t* unit_addr(const GemvParams& p, int item, int j, int* type) {
  const int tile = item >> p.split_log2, part = item & (p.split - 1);
  const GemvSeg& sg = p.seg[seg_of(p, tile)];
  *type = sg.type;
  const int ub = unit_bytes(sg.type);
  const int b = part * p.bps + j;
  return sg.w + (size_t(tile - sg.tile_begin) * p.nb + b) * ub;
}

// Streams the items item0, item0 + istride, ... (< nitems) of one warp: every
// unit is loaded one step ahead (double buffer), `flush(item, acc)` receives
// each finished item's row sums.  buf[0] must already hold the first unit
// (loaded by the caller before it waited for the previous kernel: PDL).
//
// EXACT: every item is a whole tile's K range walked in block order, and each
// row dot keeps the reference's eight lane accumulators (unit_compute_exact);
// `flush` then receives the reference's row results bit for bit.
template <int NC, int UC = UNIT_CHUNKS, bool EXACT = false, class Flush>
__device__ __forceinline__ void stream_items(const GemvParams& p, const ActSlice& act, int item0, int istride,
                                             int nitems, int lane, UnitRegsN<UC>& buf0, int first_type,
                                             Flush& flush) {
  if (item0 >= nitems) return;
  UnitRegsN<UC> buf1;
  int t0 = first_type, t1 = first_type;
  int item = item0, j = 0;
  float acc[NC];
  LaneChain lacc[EXACT ? NC : 1];
#pragma unroll
  for (int c = 0; c < NC; ++c) acc[c] = 0.0f;
#pragma unroll
  for (int c = 0; c < (EXACT ? NC : 1); ++c) lacc[c].zero();
  // One step: prefetch the unit after (item, j) into `nxt`, compute `cur`.
  // The two buffers alternate by name (no dynamic indexing, so they stay in
  // registers).
  auto step = [&](UnitRegsN<UC>& cur, int tcur, UnitRegsN<UC>& nxt, int& tnxt) -> bool {
    int nitem = item, nj = j + 1;
    if (nj == p.bps) {
      nitem = item + istride;
      nj = 0;
    }
    const bool has_next = nitem < nitems;
    if (has_next) load_unit(nxt, unit_addr(p, nitem, nj, &tnxt), tnxt, lane);
    if constexpr (EXACT) {
      unit_compute_exact<NC, UC>(cur, tcur, (item & (p.split - 1)) * p.bps + j - act.kb0, p.ncols, act, lacc);
    } else {
      unit_compute<NC, UC>(cur, tcur, (item & (p.split - 1)) * p.bps + j - act.kb0, p.ncols, act, acc);
    }
    if (nj == 0) {
      if constexpr (EXACT) {
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          acc[c] = lacc[c].total(tcur == TYPE_Q4_K);
          lacc[c].zero();
        }
      }
      flush(item, acc);
#pragma unroll
      for (int c = 0; c < NC; ++c) acc[c] = 0.0f;
    }
    item = nitem;
    j = nj;
    return has_next;
  };
  while (step(buf0, t0, buf1, t1) && step(buf1, t1, buf0, t0)) {
  }
}

// One item per warp with units 1..pre already copied into shared memory
// (`staged`, one ub_max slot per unit, completing on `bar`) and unit 0 in
// `buf0`: computes unit 0 while loading unit pre+1, then the staged units,
// then streams units pre+1 .. bps-1 through the two register buffers.  Units
// are accumulated in order 0 .. bps-1, as stream_items does.
template <int NC, int UC, class Flush>
__device__ __forceinline__ void prefetched_item(const GemvParams& p, const ActSlice& act, int item, int lane,
                                                UnitRegsN<UC>& buf0, int type, const uint8_t* staged, int ub_max,
                                                uint64_t* bar, Flush& flush) {
  float acc[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) acc[c] = 0.0f;
  const int kbase = (item & (p.split - 1)) * p.bps - act.kb0;
  UnitRegsN<UC> buf1;
  int tt;
  const int nxt = p.pre + 1;
  if (nxt < p.bps) load_unit(buf1, unit_addr(p, item, nxt, &tt), type, lane);
  unit_compute<NC, UC>(buf0, type, kbase, p.ncols, act, acc);
  if (p.pre > 0) {
    mbar_wait_parity(bar, 0, p.err);
    for (int jj = 1; jj <= p.pre; ++jj)
      unit_compute_smem<NC, UC>(staged + size_t(jj - 1) * ub_max, type, kbase + jj, p.ncols, act, acc, lane);
  }
  for (int j = nxt; j < p.bps; j += 2) {
    if (j + 1 < p.bps) load_unit(buf0, unit_addr(p, item, j + 1, &tt), type, lane);
    unit_compute<NC, UC>(buf1, type, kbase + j, p.ncols, act, acc);
    if (j + 1 < p.bps) {
      if (j + 2 < p.bps) load_unit(buf1, unit_addr(p, item, j + 2, &tt), type, lane);
      unit_compute<NC, UC>(buf0, type, kbase + j + 1, p.ncols, act, acc);
    }
  }
  flush(item, acc);
}

// Cooperative copy of the activation slice for blocks [kb0, kb0 + nblk) of
// columns [col0, col0 + ncols) into shared memory (plane A then plane B).
__device__ __forceinline__ void stage_activations(const GemvParams& p, uint8_t* dst_a, uint8_t* dst_b, int kb0,
                                                  int nblk) {
  const int nthreads = blockDim.x;
  for (int c = 0; c < p.ncols; ++c) {
    const size_t rec0 = size_t(p.col0 + c) * p.nb + kb0;
    if (dst_a) {
      const uint4* s = reinterpret_cast<const uint4*>(p.q.a + rec0 * Q8A_REC);
      uint4* d = reinterpret_cast<uint4*>(dst_a + size_t(c) * nblk * Q8A_REC);
      for (int i = threadIdx.x; i < nblk * Q8A_REC / 16; i += nthreads) d[i] = __ldg(s + i);
    }
    if (dst_b) {
      const uint4* s = reinterpret_cast<const uint4*>(p.q.b + rec0 * Q8B_REC);
      uint4* d = reinterpret_cast<uint4*>(dst_b + size_t(c) * nblk * Q8B_REC);
      for (int i = threadIdx.x; i < nblk * Q8B_REC / 16; i += nthreads) d[i] = __ldg(s + i);
    }
  }
}

// Thread 0 copies the CTA's activation slice (the Q8_K records of blocks
// [kb0, kb0 + nblk) of every column, contiguous per column and plane) into
// shared memory with bulk copies completing on `bar`, which it initializes;
// the caller syncs the CTA before anyone waits on `bar`.  One L2 round trip
// instead of a load/store loop.
__device__ __forceinline__ void stage_activations_bulk(const GemvParams& p, uint8_t* dst_a, uint8_t* dst_b, int kb0,
                                                       int nblk, uint64_t* bar) {
  if (threadIdx.x != 0) return;
  const uint32_t per_col = uint32_t(nblk) * uint32_t((dst_a ? Q8A_REC : 0) + (dst_b ? Q8B_REC : 0));
  mbar_init(bar, 1);
  mbar_expect_tx(bar, per_col * uint32_t(p.ncols));
  for (int c = 0; c < p.ncols; ++c) {
    const size_t rec0 = size_t(p.col0 + c) * p.nb + kb0;
    if (dst_a) bulk_copy_g2s(dst_a + size_t(c) * nblk * Q8A_REC, p.q.a + rec0 * Q8A_REC, uint32_t(nblk * Q8A_REC), bar);
    if (dst_b) bulk_copy_g2s(dst_b + size_t(c) * nblk * Q8B_REC, p.q.b + rec0 * Q8B_REC, uint32_t(nblk * Q8B_REC), bar);
  }
}

__host__ __device__ inline void gemv_planes(const GemvParams& p, bool* need_a, bool* need_b) {
  *need_a = *need_b = false;
  if (p.pro.mode != GEMV_PRO_NONE) {  // the prologue's quantizer writes both planes
    *need_a = *need_b = true;
    return;
  }
  for (int i = 0; i < p.nseg; ++i) {
    if (p.seg[i].type == TYPE_Q4_K) *need_a = true;
    else *need_b = true;
  }
}

// Dynamic shared memory of a launch: the activation slice of one CTA.
__host__ __device__ inline size_t gemv_smem_bytes(const GemvParams& p, int nblk) {
  bool a, b;
  gemv_planes(p, &a, &b);
  return size_t(p.ncols) * nblk * ((a ? Q8A_REC : 0) + (b ? Q8B_REC : 0));
}

}  // namespace hc
