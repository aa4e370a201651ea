// hc_kernels.cuh -- launchers shared between the kernel files and the C ABI.
#pragma once
#include <mutex>
#include <utility>
#include <vector>

#include "hc_common.cuh"

namespace hc {

constexpr int GEMV_WARPS = 4;  // warps per CTA; each warp owns whole blocks
constexpr int GEMV_BPW = 2;    // blocks per warp per round (loads issued together)
constexpr int GEMV_MAXSEG = 8; // weights sharing one input in one launch

struct GemvSeg {
  const uint8_t* w;  // tile layout
  float* out;        // out[col * rows + row]
  int type;
  int rows;
  int tile_begin;    // first global tile index of this segment
  int pad;
};

// Fused input of a matmul whose input is an RMSNorm of the residual stream
// (the per-layer hc_norm_quant_kernel folded into the GEMV): every CTA computes
// the norm of the whole D = 2048 vector itself and quantizes the 256-blocks
// of its K slice straight into its shared-memory activation records.
enum { GEMV_PRO_NONE = 0, GEMV_PRO_NORM = 1, GEMV_PRO_RESID_NORM = 2, GEMV_PRO_QUANT = 3 };
struct GemvPrologue {
  int mode;
  int pad_;
  const float* x;       // residual stream [col][2048]
  const float* y;       // RESID_NORM: projection output added after its own norm [col][2048]
  const float* w_post;  // RESID_NORM: that norm's weight
  const float* w_pre;   // weight of the norm of this matmul's input
  float* x_out;         // RESID_NORM: CTA 0 stores x + rmsnorm(y) * w_post here (not x: other CTAs read x)
  double eps;
};
constexpr int GEMV_PRO_D = 2048;

struct GemvParams {
  GemvSeg seg[GEMV_MAXSEG];
  int nseg;
  int K, nb;        // input size and 256-blocks per row
  int split;        // K parts per tile (1, 2, 4, or 8..32 = a cluster of split/4 CTAs)
  int split_log2;   // log2(split)
  int bps;          // blocks per part = nb / split
  int col0, ncols;  // this launch covers columns [col0, col0 + ncols), ncols <= 8
  int total_tiles;  // over all segments
  int bulk;         // 1: each CTA copies all of its units into shared memory up front
  int q4small;      // 1: every weight is Q4_K and ncols <= 2 (Q4_K-sized register buffers, 4 CTAs per SM)
  int pre;          // streaming mode, one item per warp: units 1..pre of the item are copied into shared
                    // memory before the wait for the previous kernel (0: only unit 0, into registers)
  int ring;         // tensor-core GEMV (hc_gemv_mma.cu): weight-unit slots per warp
  int* err;         // device status word (bounded-wait timeouts)
  Q8Buf q;
  GemvPrologue pro; // mode != NONE: activations computed by every CTA instead of read from q
};

// Device status word of the current device (hc_api.cu).
int* device_status_word();

constexpr int GEMV_WARPS_PER_CTA = 4;
constexpr int GEMV_THREADS = GEMV_WARPS_PER_CTA * 32;
constexpr int GEMV_CTAS_PER_SM = 3;
constexpr int GEMV_CTAS_PER_SM_Q4 = 4;  // Q4_K-only launches of <= 2 columns (smaller register buffers)
constexpr int GEMV_MAX_SMEM = 200 * 1024;
constexpr int GEMV_BULK_MAX_UNITS_SMEM = 112 * 1024;  // unit bytes a bulk-mode CTA may stage
constexpr int GEMV_SM_SMEM = 228 * 1024;              // shared memory per SM
constexpr int GEMV_MAX_CLUSTER = 8;                   // CTAs per tile at split 32
constexpr int GEMV_PRE_SM_SMEM = 160 * 1024;          // shared memory per SM a streaming launch may fill
                                                      // with prefetched units (the rest serves the kernels
                                                      // launched after it)

// Static shared memory of hc_gemv_kernel for a launch of `ncols` columns (the
// column count rounds up to the kernel's 1/2/4/8 template): the per-warp
// partials, rank 0's cluster gather array and the two mbarriers.
inline size_t gemv_static_smem(int ncols) {
  const int nc = ncols <= 1 ? 1 : ncols <= 2 ? 2 : ncols <= 4 ? 4 : 8;
  return size_t(GEMV_WARPS_PER_CTA + GEMV_MAX_CLUSTER) * nc * 32 * 4 + GEMV_WARPS_PER_CTA * 256 + 128;
}

__host__ __device__ inline int unit_bytes(int type) { return int(tile_block_bytes(type)); }

// Asks for the maximal shared-memory carveout for kernel `fn` (once per
// device), so its CTAs, launched early under programmatic dependent launch,
// can join SMs that still run the previous kernel without those SMs first
// draining to change their L1 / shared-memory split.
inline void use_max_carveout(const void* fn) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  static std::mutex mu;
  static std::vector<std::pair<const void*, int>> done;
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& d : done)
    if (d.first == fn && d.second == dev) return;
  cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
  done.emplace_back(fn, dev);
}

cudaError_t launch_q8k_quantize(const float* x, int K, int cols, const Q8Buf& q, int8_t* nat_qs, int16_t* nat_bs32,
                                float* nat_d, cudaStream_t stream);
cudaError_t launch_repack(int type, const uint8_t* src, uint8_t* dst, int rows, int rows_pad, int nb,
                          cudaStream_t stream);
cudaError_t launch_dequant(int type, const uint8_t* w, float* out, int rows, int nb, cudaStream_t stream);
// hp_matmul_dequantized_f32 arithmetic on a resident (tile-layout) weight:
// out[col * rows + row], one sequential f32 chain per (row, column).
cudaError_t launch_dequant_matmul(int type, const uint8_t* w, int nb, int rows, int rows_pad, const float* x, int K,
                                  int cols, float* out, cudaStream_t stream);

// Picks the K split for a launch; fills p.split and p.bps.
void gemv_plan(GemvParams& p);
// Grid size of a launch planned by gemv_plan.
int gemv_grid(const GemvParams& p);
int sm_count();
// Persistent grid over `items` items, one warp per item at a time: the fewest
// CTAs (<= cap) that give every warp the same number of items.
int persistent_grid(int items, int cap);
int persistent_grid_w(int items, int cap, int warps_per_cta);
cudaError_t launch_gemv(const GemvParams& p, cudaStream_t stream);

// Exact-order matmul (hc_gemvx.cu): every row dot equals the reference's
// vec_dot_q*_k_q8_k_prepared bit for bit (its 8 f32 lane accumulators in
// block order).  Same segments / outputs / Q8_K workspace as GemvParams.
constexpr int GEMVX_MAX_COLS = 8;
struct GemvxParams {
  GemvSeg seg[GEMV_MAXSEG];
  int nseg;
  int K, nb;         // input size and 256-blocks per row
  int C;             // CTAs per tile (one cluster) splitting its K range
  int nbc;           // blocks per CTA = nb / C
  int col0, ncols;   // columns [col0, col0 + ncols), ncols <= GEMVX_MAX_COLS
  int total_tiles;   // over all segments
  int R;             // ring slots per warp
  int slot;          // bytes per ring slot (the largest unit)
  int planes;        // activation planes the weight types read: 1 = A (Q4_K), 2 = B (Q6_K)
  int* err;          // device status word (bounded-wait timeouts)
  Q8Buf q;
  // mode != NONE: every CTA computes its activation records itself from
  // pro.x (width GEMV_PRO_D): NORM / RESID_NORM as the GEMV prologue of the
  // reordered step, QUANT = Q8_K of pro.x as it is (x_out, y, w_* unused)
  GemvPrologue pro;
};
// Fills C, nbc, R, slot, err; returns the grid size (<= 0: no plan fits).
int gemvx_plan(GemvxParams& p, int sms);
// The warp-per-tile form (rows of at most 16 blocks): returns the columns per
// warp (0: the form does not apply) and the grid size in *grid.
int gemvw_plan(GemvxParams& p, int sms, int* grid, bool any_size = false);
cudaError_t launch_gemvx(GemvxParams& p, cudaStream_t st);

// L2 prefetch of up to PREFETCH_MAX_RANGES byte ranges (hc_prefetch.cu):
// cp.async.bulk.prefetch.L2 over each range, 16-byte aligned starts.
constexpr int PREFETCH_MAX_RANGES = 8;
struct PrefetchList {
  const void* ptr[PREFETCH_MAX_RANGES];
  size_t bytes[PREFETCH_MAX_RANGES];
  int n;
};
cudaError_t launch_l2_prefetch(const PrefetchList& l, cudaStream_t st);

// Inputs of at least TC_MIN_COLS columns go to the tensor-core matmul
// (hc_gemm_tc.cu), one launch per weight covering every column.
constexpr int TC_MIN_COLS = 16;
// Inputs of GEMV_MMA_MIN_COLS .. 8 columns go to the tensor-core GEMV
// (hc_gemv_mma.cu); fewer to the dp4a GEMV.
constexpr int GEMV_MMA_MIN_COLS = 3;
cudaError_t launch_gemv_mma(GemvParams& p, cudaStream_t stream);
cudaError_t launch_gemm_tc(const GemvSeg& seg, int nb, const Q8Buf& q, int col0, int ncols, cudaStream_t st);
// The same product for Q4_K on tcgen05 (hc_gemm_t5.cu); HPC_GEMM_T5=1 routes
// launch_gemm_tc's Q4_K launches here.
bool gemm_t5_enabled();
void set_gemm_t5(bool on);
cudaError_t launch_gemm_t5(const GemvSeg& seg, int nb, const Q8Buf& q, int col0, int ncols, cudaStream_t st);

}  // namespace hc
