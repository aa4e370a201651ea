// hc_persist.cuh -- plan and launch interface of the persistent decode-step
// kernel (hc_persist.cu): all decoder layers of one M = 1 step in a single
// cooperative launch.
#pragma once
#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

#include "hc_common.cuh"

namespace hc {

constexpr int P_WARPS = 8;                      // warps per CTA
constexpr int P_THREADS = 32 * P_WARPS;
constexpr int P_SLOTS = 3;                      // ring slots per warp
constexpr int P_SLOT_BYTES = 8192;              // >= one Q6_K tile-block (6720 B) or one attention unit
constexpr int P_ATT_TOK = 4;                    // KV tokens per attention unit (4 K + 4 V rows of 1 KB)
constexpr int P_ATT_WARPS = 4;                  // warps per CTA that run attention units
constexpr int P_WARP_TILES = 4;                 // 32-row tiles one warp's unit range may touch
constexpr int P_MAXSEG = 8;                     // per-CTA partials of one tile (host-checked)
constexpr int P_MAX_G = 4;                      // query heads per KV head
constexpr int P_ATT_REC = 2 * P_MAX_G + P_MAX_G * 256;  // floats per attention partial: m[G], l[G], o[G][256]
constexpr int P_ACT_BYTES = 64 * Q8B_REC;       // activation records staged per CTA (up to 16384 wide)

// Counters per layer, in stage order; each in its own 128-byte line.
enum PStage { PS_QKV = 0, PS_ATT, PS_COMB, PS_O, PS_GU, PS_ACT, PS_DOWN, PS_COUNT };
constexpr int P_CTR_STRIDE = 32;

// One GEMV stage: up to three weights sharing one input (tile ranges
// concatenated), K = 256 * B.  Its output is per-CTA partial row sums:
// part[(tile * maxseg + seg) * 32 + row], seg = CTA index - first CTA of the
// tile's units.
struct PGemv {
  const uint8_t* w[3];
  int type[3];
  int tile_end[3];  // cumulative tile counts
  int nseg;
  int B;            // 256-blocks per row
  int tiles;        // total tiles
  int maxseg;
  float* part;
};

struct PLayer {
  PGemv qkv, o, gu, down;
  const float *n_attn, *n_q, *n_k, *n_post_attn, *n_ffn, *n_post_ffw;
  float* kc;  // K [cap][KVH][256] of the layer's KV source
  float* vc;  // V [cap][KVH][256]
  int own_kv;
  int pad_;
};

struct PParams {
  const PLayer* layers;
  int nlayers, D, F, H, KVH, cap;
  double eps;
  const int32_t* pos;
  const double* cos_t;
  const double* sin_t;
  float* X;           // residual stream x_l (written by CTA 0), final residual on exit
  float* H1;          // post-attention residual of the current layer (written by CTA 0)
  uint8_t* q8_attn;   // Q8_K records of the attention vector (q8buf_carve(base, H*256, 1))
  uint8_t* q8_act;    // Q8_K records of the FFN activation (q8buf_carve(base, F, 1))
  float* att_part;    // [grid][P_ATT_REC]
  unsigned* counters; // [nlayers][PS_COUNT] x P_CTR_STRIDE, zero at launch
  unsigned* kvh_counters;  // [nlayers][KVH] attention CTAs done per KV head, zero at launch
  unsigned* blk_counters;  // [nlayers][F/256] gate/up producers done per activation block, zero at launch
  int* abort_word;    // zero at launch; set when any wait gives up
  int* err;           // device status word (HPC_ERR_TIMEOUT on a timeout)
};

// CTA range of a stage's U units: [U*c/G, U*(c+1)/G) (U * G < 2^31, host-checked).
__host__ __device__ inline int p_range_lo(int U, int c, int G) { return int(unsigned(U) * unsigned(c) / unsigned(G)); }
// The CTA whose range holds unit u.
__host__ __device__ inline int p_cta_of(int u, int U, int G) {
  return int((unsigned(u + 1) * unsigned(G) - 1u) / unsigned(U));
}

size_t persist_smem_bytes();
// Largest per-tile segment count of a GEMV stage of `tiles` tiles x B blocks
// over `grid` CTAs, and whether every warp range touches <= P_WARP_TILES tiles.
int persist_maxseg(int tiles, int B, int grid, bool* warp_tiles_ok);
// Grid size of the persistent launch on the current device (0 if it cannot be co-resident).
int persist_grid();
cudaError_t launch_persistent_step(const PParams& p, int grid, cudaStream_t st);

}  // namespace hc
