// hc_gemm_t5.cu -- Q4_K x Q8_K matmul on the fifth-generation tensor cores
// (tcgen05.mma kind::i8, accumulators in tensor memory) for wide inputs:
// prefill's Q4_K projections.
//
// The arithmetic is vec_dot_q4_k_q8_k's (lib.rs:2117-2172), the same as the
// mma.sync matmul's (hc_gemm_tc.cu): per (row, column, 256-block) the exact
// int32 sum over the eight 32-element groups of sc_g * dot_g, combined with
// d, dmin and the activation's d in f32 once per block.  The K-quant scale
// multiplies each group's dot before the groups are added, which a tensor
// core accumulator cannot do by itself; here the 6-bit scale is split,
// sc = 8 s1 + s0 with s0, s1 in 0..7, and the A operand is the weights
// pre-multiplied by each half: q * s0 and q * s1 are at most 105, so both
// fit int8, and one pair of MMAs per group accumulates
//   D0 = sum_g sum_k (q s0) a,   D1 = sum_g sum_k (q s1) a
// over the whole 256-block in tensor memory; the block sum is D0 + 8 D1,
// exact in int32 (|D| < 8 * 32 * 105 * 128).
//
// CTA = 128 weight rows (four row tiles) x 64 columns, 8 warps.  Per
// 256-block: the four weight units and the 64 columns' Q8_K records arrive
// by cp.async (the records straight into the B operand's layout); every
// thread builds its row's A0 / A1 words for the eight groups (packed-byte
// multiplies: four weights per instruction; two threads per row) in the
// K-major canonical layout
// without swizzle (8-row x 16-byte core matrices, 128 bytes between the two
// K halves, 256 bytes between row groups); thread 0 issues the 16 MMAs
// (M=128, N=64, K=32) and commits them to an mbarrier; then every warp reads
// its 32 rows x 32 columns of D0 / D1 from tensor memory (warps w and w + 4
// share lane quarter w % 4) and does the f32 combine.  Blocks are pipelined:
// block b's MMAs run while block b - 1's combine and block b + 2's copies
// proceed.
// Within a group, A and B use the same permutation of the 32 elements (the
// row-tile words and the plane-A record words hold the same accumulator
// lanes), which a dot product does not see.
#include <atomic>
#include <cstdlib>

#include "hc_bulk.cuh"
#include "hc_common.cuh"
#include "hc_kernels.cuh"
#include "hc_unpack.cuh"

namespace hc {

namespace {

constexpr int T5_ROWS = 128;     // 4 row tiles
constexpr int T5_COLS = 64;      // MMA N
constexpr int T5_THREADS = 256;  // 8 warps: warp w = TMEM lanes 32 (w % 4) .. + 31 = tile w % 4, columns 32 (w / 4) ..
constexpr int T5_HCOLS = T5_COLS / 2;  // columns per warp in the epilogue
constexpr int T5_UB = 4608;      // Q4_K unit bytes
constexpr int T5_GROUP_A = T5_ROWS * 32;  // bytes of one group's A operand (128 rows x 32)
constexpr int T5_GROUP_B = T5_COLS * 32;  // bytes of one group's B operand (64 columns x 32)
constexpr int T5_TMEM_COLS = 256;         // two sets of D0 (64 columns) + D1 (64 columns)

// shared memory (bytes): two unit slots, two A0/A1 sets (the tensor core
// reads set b % 2 while set (b + 1) % 2 is built), three B + record-tail
// slots (block b's MMAs, block b - 1's epilogue and block b + 1's copies in
// flight at once)
constexpr int T5_UNITS = 4 * T5_UB;                          // 18432
constexpr int T5_A = 2 * 8 * T5_GROUP_A;                     // A0 then A1: 65536
constexpr int T5_BT = 8 * T5_GROUP_B + T5_COLS * 32;         // B then tails: 18432
constexpr int T5_OFF_UNITS = 0;
constexpr int T5_OFF_A = T5_OFF_UNITS + 2 * T5_UNITS;        // 36864
constexpr int T5_OFF_BT = T5_OFF_A + 2 * T5_A;               // 167936
constexpr int T5_SMEM = T5_OFF_BT + 3 * T5_BT;               // 223232
constexpr int T5_TMEM_SETS = 2;                              // D0/D1 of blocks b and b - 1

struct T5Params {
  const uint8_t* w;    // Q4_K row tiles
  const uint8_t* act;  // Q8_K plane A records, [col][nb]
  float* out;          // out[col * rows + row]
  int rows, tiles, nb, ncols, col0;
  int* err;
};

// byte offset of (row or column mn, byte k of the 32-byte group) in a
// K-major, unswizzled operand: core matrices of 8 x 16 bytes
__device__ __forceinline__ int t5_off(int mn, int khalf) { return (mn >> 3) * 256 + khalf * 128 + (mn & 7) * 16; }

// shared-memory matrix descriptor (tcgen05): start address, leading byte
// offset 128 (between the two K halves), stride byte offset 256 (between
// 8-row groups), descriptor version 1, no swizzle
__device__ __forceinline__ uint64_t t5_desc(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3fff) | (uint64_t(128 >> 4) << 16) | (uint64_t(256 >> 4) << 32) | (1ull << 46);
}

// instruction descriptor: s32 accumulator, s8 x s8, both K-major, N = 64, M = 128
constexpr uint32_t T5_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(T5_COLS >> 3) << 17) |
                              (uint32_t(T5_ROWS >> 4) << 24);

__device__ __forceinline__ void t5_mma(uint32_t d_tmem, uint64_t a, uint64_t b, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(T5_IDESC), "r"(uint32_t(accumulate)), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void t5_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__global__ void __launch_bounds__(T5_THREADS, 1) hc_gemm_t5_kernel(const __grid_constant__ T5Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t mma_bar[T5_TMEM_SETS];
  __shared__ uint32_t tmem_slot;
  const int t = int(threadIdx.x), warp = t >> 5, lane = t & 31;
  const int tile0 = int(blockIdx.x) * 4, col0 = p.col0 + int(blockIdx.y) * T5_COLS;
  const uint32_t sbase = smem_u32(smem);
  if (warp == 0) {  // tensor memory for two D0 / D1 sets
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(uint32_t(T5_TMEM_COLS))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (t == 0)
    for (int s = 0; s < T5_TMEM_SETS; ++s) mbar_init(&mma_bar[s], 1);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;
  // copies of block b: its four units into unit slot b % 2, its records into
  // B/tail slot b % 3 (two 16-byte pieces per group, straight into the B
  // operand's layout); one cp.async group per block
  auto issue = [&](int b) {
    if (b < p.nb) {
      uint8_t* us = smem + T5_OFF_UNITS + (b & 1) * T5_UNITS;
      for (int i = t; i < 4 * T5_UB / 16; i += T5_THREADS) {
        const int u = i / (T5_UB / 16), o = i % (T5_UB / 16);
        const int tile = min(tile0 + u, p.tiles - 1);
        cp_async16(us + u * T5_UB + o * 16, p.w + (size_t(tile) * p.nb + b) * T5_UB + o * 16);
      }
      uint8_t* bt = smem + T5_OFF_BT + (b % 3) * T5_BT;
      for (int i = t; i < T5_COLS * 18; i += T5_THREADS) {  // 18 pieces per 288-byte record
        const int n = i / 18, piece = i % 18;
        const int col = min(col0 + n, p.col0 + p.ncols - 1);
        const uint8_t* rec = p.act + (size_t(col) * p.nb + b) * Q8A_REC;
        if (piece < 16) cp_async16(bt + (piece >> 1) * T5_GROUP_B + t5_off(n, piece & 1), rec + 16 * piece);
        else cp_async16(bt + 8 * T5_GROUP_B + n * 32 + 16 * (piece - 16), rec + 16 * piece);
      }
    }
    cp_async_commit();  // empty past the last block: the group count stays uniform
  };
  const int quarter = warp & 3, part = warp >> 2;  // TMEM lane quarter = row tile; column half / pair half
  float acc[T5_HCOLS];
#pragma unroll
  for (int n = 0; n < T5_HCOLS; ++n) acc[n] = 0.0f;
  const int row = quarter * 32 + lane;  // this thread's row of the CTA (tile `quarter`, lane = row in the tile)
  bool ok = true;
  // block b's f32 combine: this warp's 32 rows, its 32 columns of D0 / D1,
  // and the records' tails
  auto epilogue = [&](int b, const Q4KHeader& h) {
    const uint32_t set = uint32_t(b & 1) * 2 * T5_COLS, lane_base = uint32_t(quarter * 32) << 16;
    const uint8_t* tails = smem + T5_OFF_BT + (b % 3) * T5_BT + 8 * T5_GROUP_B;
    {
      uint32_t r0[32], r1[32];
      t5_ld32(tmem + lane_base + set + T5_HCOLS * part, r0);
      t5_ld32(tmem + lane_base + set + T5_COLS + T5_HCOLS * part, r1);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = T5_HCOLS * part + j;
        const uint8_t* tail = tails + n * 32;
        const uint4 bs = *reinterpret_cast<const uint4*>(tail + (Q8A_BS - 256));
        const float d8 = *reinterpret_cast<const float*>(tail + (Q8A_D - 256));
        int ms = __dp2a_lo(int(bs.x), int(h.mn_lo), 0);
        ms = __dp2a_hi(int(bs.y), int(h.mn_lo), ms);
        ms = __dp2a_lo(int(bs.z), int(h.mn_hi), ms);
        ms = __dp2a_hi(int(bs.w), int(h.mn_hi), ms);
        const int isum = int(r0[j]) + 8 * int(r1[j]);
        acc[j] += __fmul_rn(h.d, d8) * float(isum) - __fmul_rn(h.dmin, d8) * float(ms);
      }
    }
  };
  issue(0);
  issue(1);
  Q4KHeader prev_hd{};
  for (int b = 0; b < p.nb; ++b) {
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // block b landed (b + 1 may still fly)
    __syncthreads();
    // A0 / A1 of block b into set b % 2 (the MMAs of block b - 2 read it
    // and finished before block b - 1's epilogue)
    const uint8_t* unit = smem + T5_OFF_UNITS + (b & 1) * T5_UNITS + quarter * T5_UB;
    const Q4KHeader hd = q4k_header(*reinterpret_cast<const uint4*>(unit + lane * 16));
    uint8_t* aset = smem + T5_OFF_A + (b & 1) * T5_A;
#pragma unroll
    for (int pi = 0; pi < 2; ++pi) {  // this thread's two of the row's four quant pairs
      const int pp = 2 * part + pi;
      const uint4 u0 = *reinterpret_cast<const uint4*>(unit + (1 + 2 * pp) * 512 + lane * 16);
      const uint4 u1 = *reinterpret_cast<const uint4*>(unit + (2 + 2 * pp) * 512 + lane * 16);
      const uint32_t wd[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
      for (int hi = 0; hi < 2; ++hi) {
        const int g = 2 * pp + hi, sc = hd.sc(g);
        const uint32_t s0 = uint32_t(sc & 7), s1 = uint32_t(sc >> 3);
        uint32_t a0[8], a1[8];
#pragma unroll
        for (int l = 0; l < 8; ++l) {
          const uint32_t q = hi ? (wd[l] >> 4) & 0x0f0f0f0fu : wd[l] & 0x0f0f0f0fu;
          a0[l] = q * s0;  // four bytes at once: each product <= 105, no carry between bytes
          a1[l] = q * s1;
        }
        uint8_t* d0 = aset + g * T5_GROUP_A;
        uint8_t* d1 = aset + (8 + g) * T5_GROUP_A;
        *reinterpret_cast<uint4*>(d0 + t5_off(row, 0)) = make_uint4(a0[0], a0[1], a0[2], a0[3]);
        *reinterpret_cast<uint4*>(d0 + t5_off(row, 1)) = make_uint4(a0[4], a0[5], a0[6], a0[7]);
        *reinterpret_cast<uint4*>(d1 + t5_off(row, 0)) = make_uint4(a1[0], a1[1], a1[2], a1[3]);
        *reinterpret_cast<uint4*>(d1 + t5_off(row, 1)) = make_uint4(a1[4], a1[5], a1[6], a1[7]);
      }
    }
    // the operands were written by the generic proxy; the tensor core reads
    // them through the async proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (t == 0 && ok) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t set = uint32_t(b & 1) * 2 * T5_COLS;
      const uint32_t bsm = sbase + T5_OFF_BT + (b % 3) * T5_BT, asm_ = sbase + T5_OFF_A + (b & 1) * T5_A;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const uint64_t db = t5_desc(bsm + g * T5_GROUP_B);
        t5_mma(tmem + set, t5_desc(asm_ + g * T5_GROUP_A), db, g > 0);
        t5_mma(tmem + set + T5_COLS, t5_desc(asm_ + (8 + g) * T5_GROUP_A), db, g > 0);
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(&mma_bar[b & 1]))
                   : "memory");
    }
    // block b - 1: its MMAs ran while block b was built
    if (b > 0) {
      if (ok && !mbar_wait_parity(&mma_bar[(b - 1) & 1], uint32_t(((b - 1) >> 1) & 1), p.err)) ok = false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (ok) epilogue(b - 1, prev_hd);
    }
    prev_hd = hd;
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();  // block b - 1's records, D set and unit slot are free
    issue(b + 2);
  }
  if (ok && !mbar_wait_parity(&mma_bar[(p.nb - 1) & 1], uint32_t(((p.nb - 1) >> 1) & 1), p.err)) ok = false;
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (ok) epilogue(p.nb - 1, prev_hd);
  asm volatile("cp.async.wait_all;" ::: "memory");
  const int orow = (tile0 + quarter) * TILE + lane;
  if (ok && tile0 + quarter < p.tiles && orow < p.rows) {
#pragma unroll
    for (int j = 0; j < T5_HCOLS; ++j) {
      const int n = T5_HCOLS * part + j;
      if (col0 + n < p.col0 + p.ncols) p.out[size_t(col0 + n) * p.rows + orow] = acc[j];
    }
  }
  // after a timeout, the MMAs still in flight get one more bounded wait
  // before the tensor memory is freed
  if (!ok)
    for (int s = 0; s < T5_TMEM_SETS; ++s) mbar_wait_parity(&mma_bar[s], 0, nullptr);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(uint32_t(T5_TMEM_COLS))
                 : "memory");
}

}  // namespace

// hpc_set_wide_matmul_kind(1) (or HPC_GEMM_T5=1 at load) routes the wide
// Q4_K matmul to this kernel.
static std::atomic<int> g_t5{-1};
bool gemm_t5_enabled() {
  int v = g_t5.load();
  if (v < 0) {
    const char* e = getenv("HPC_GEMM_T5");
    v = e && atoi(e) != 0 ? 1 : 0;
    g_t5.store(v);
  }
  return v == 1;
}
void set_gemm_t5(bool on) { g_t5.store(on ? 1 : 0); }

cudaError_t launch_gemm_t5(const GemvSeg& seg, int nb, const Q8Buf& q, int col0, int ncols, cudaStream_t st) {
  if (seg.type != TYPE_Q4_K) return cudaErrorInvalidValue;
  T5Params p;
  p.w = seg.w;
  p.act = q.a;
  p.out = seg.out;
  p.rows = seg.rows;
  p.tiles = (seg.rows + TILE - 1) / TILE;
  p.nb = nb;
  p.ncols = ncols;
  p.col0 = col0;
  p.err = device_status_word();
  static std::atomic<uint64_t> attr{0};
  const cudaError_t ea = once_per_current_device(attr, [] {
    return cudaFuncSetAttribute(hc_gemm_t5_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, T5_SMEM);
  });
  if (ea != cudaSuccess) return ea;
  const dim3 grid(unsigned((p.tiles + 3) / 4), unsigned((ncols + T5_COLS - 1) / T5_COLS));
  hc_gemm_t5_kernel<<<grid, T5_THREADS, T5_SMEM, st>>>(p);
  return cudaGetLastError();
}

}  // namespace hc
