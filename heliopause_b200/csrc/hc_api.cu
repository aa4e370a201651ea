// hc_api.cu -- the C ABI declared in include/heliocuda.h.
//
// Validation order and status codes follow the WASM drivers they replace
// (packages/engine/wasm-kernels/src/lib.rs:41-426): the input/output length
// check comes first (ERR_SHAPE), then the type/row-size check (ERR_TYPE),
// then the weight length (ERR_SHAPE).  A resident handle carries its own
// shape, so "weight length" becomes "handle shape equals (input_size,
// row_count)".
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/heliocuda.h"
#include "hc_common.cuh"
#include "hc_internal.h"
#include "hc_kernels.cuh"
#include "hc_lmhead.cuh"

thread_local std::string g_last_error;

int hpc_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int hpc_cuda_fail(cudaError_t e, const char* what) {
  return hpc_fail(HPC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

namespace {

int (*const fail)(int, const char*, ...) = hpc_fail;
int (*const cuda_fail)(cudaError_t, const char*) = hpc_cuda_fail;

bool supported_type(int t) { return t == HPC_TYPE_Q4_K || t == HPC_TYPE_Q6_K; }

// lib.rs:1551-1561 quantized_row_bytes for every reference type id.
bool row_bytes(int type, size_t k, size_t* out) {
  switch (type) {
    case HPC_TYPE_Q4_K: if (k % 256) return false; *out = k / 256 * 144; return true;
    case HPC_TYPE_Q5_K: if (k % 256) return false; *out = k / 256 * 176; return true;
    case HPC_TYPE_Q6_K: if (k % 256) return false; *out = k / 256 * 210; return true;
    case HPC_TYPE_IQ4_XS: if (k % 256) return false; *out = k / 256 * 136; return true;
    case HPC_TYPE_Q8_0: if (k % 32) return false; *out = k / 32 * 34; return true;
    case HPC_TYPE_Q4_0: if (k % 32) return false; *out = k / 32 * 18; return true;
    default: return false;
  }
}

bool mul_overflows(size_t a, size_t b, size_t* out) {
  if (a != 0 && b > SIZE_MAX / a) return true;
  *out = a * b;
  return false;
}

}  // namespace

static bool valid(const hpc_weight_s* h) { return hpc_weight_valid(h); }

// One status word per device for bounded-wait timeouts inside kernels.
static __device__ int g_status_word;

namespace hc {
int* device_status_word() {
  static std::mutex mu;
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) == cudaSuccess) ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}
}  // namespace hc

// Order of the public matmul / LM-head entry points (hpc_set_matmul_order):
// true = the reference's f32 order (the default), false = the reordered kernels.
static std::atomic<bool> g_exact_order{true};

extern "C" {

const char* hpc_last_error(void) { return g_last_error.c_str(); }

int hpc_version(void) { return (1 << 16) | 0; }

int hpc_device_error(void) {
  int* w = hc::device_status_word();
  if (!w) return fail(HPC_ERR_CUDA, "no device status word");
  int v = 0;
  HPC_CK(cudaMemcpy(&v, w, sizeof v, cudaMemcpyDeviceToHost), "read device status");
  if (v == 0) return HPC_OK;
  const int zero = 0;
  HPC_CK(cudaMemcpy(w, &zero, sizeof zero, cudaMemcpyHostToDevice), "clear device status");
  return fail(HPC_ERR_TIMEOUT, "a kernel wait timed out on the device (code %d)", v);
}

int hpc_device_init(int device) {
  int n = 0;
  HPC_CK(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
  if (device < 0 || device >= n) return fail(HPC_ERR_ARG, "device %d out of range (%d devices)", device, n);
  HPC_CK(cudaSetDevice(device), "cudaSetDevice");
  cudaDeviceProp prop;
  HPC_CK(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major != 10) return fail(HPC_ERR_CUDA, "device %d is sm_%d%d; this library is built for sm_100a", device,
                                    prop.major, prop.minor);
  return HPC_OK;
}

static int upload_common(int type_id, const void* src, bool src_on_device, size_t byte_len, size_t input_size,
                         size_t row_count, cudaStream_t stream, hpc_weight* out_handle) {
  if (!out_handle) return fail(HPC_ERR_ARG, "null out_handle");
  *out_handle = nullptr;
  size_t rb;
  if (!row_bytes(type_id, input_size, &rb)) return fail(HPC_ERR_TYPE, "weight upload: unsupported type %d / input size %zu", type_id, input_size);
  if (!supported_type(type_id)) return fail(HPC_ERR_TYPE, "weight upload: type %d is not resident on the GPU (Q4_K and Q6_K only)", type_id);
  size_t want;
  if (input_size == 0 || row_count == 0 || mul_overflows(rb, row_count, &want) || byte_len != want)
    return fail(HPC_ERR_SHAPE, "weight upload shape mismatch: %zu bytes for %zu rows of %zu", byte_len, row_count, input_size);
  if (!src) return fail(HPC_ERR_ARG, "null weight bytes");
  if (row_count > (size_t(1) << 30) || input_size > (size_t(1) << 24))
    return fail(HPC_ERR_SHAPE, "weight upload: shape too large");
  int dev = 0;
  HPC_CK(cudaGetDevice(&dev), "cudaGetDevice");
  const int nb = int(input_size / 256);
  const size_t rows_pad = (row_count + hc::TILE - 1) / hc::TILE * hc::TILE;
  const size_t bytes = rows_pad / hc::TILE * size_t(nb) * hc::tile_block_bytes(type_id);
  uint8_t* d_data = nullptr;
  uint8_t* d_raw = nullptr;
  HPC_CK(cudaMalloc(&d_data, bytes), "cudaMalloc(weight)");
  const uint8_t* raw = static_cast<const uint8_t*>(src);
  cudaError_t e = cudaSuccess;
  if (!src_on_device) {
    e = cudaMalloc(&d_raw, byte_len);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_raw, src, byte_len, cudaMemcpyHostToDevice, stream);
    raw = d_raw;
  }
  if (e == cudaSuccess) e = hc::launch_repack(type_id, raw, d_data, int(row_count), int(rows_pad), nb, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (d_raw) cudaFree(d_raw);
  if (e != cudaSuccess) {
    cudaFree(d_data);
    return cuda_fail(e, "weight upload/repack");
  }
  auto* h = new hpc_weight_s;
  h->magic = kWeightMagic;
  h->type = type_id;
  h->device = dev;
  h->input_size = input_size;
  h->row_count = row_count;
  h->rows_pad = rows_pad;
  h->nb = nb;
  h->d_data = d_data;
  h->bytes = bytes;
  *out_handle = h;
  return HPC_OK;
}

int hpc_weight_upload(int type_id, const uint8_t* host_bytes, size_t byte_len, size_t input_size, size_t row_count,
                      hpc_weight* out_handle) {
  return upload_common(type_id, host_bytes, false, byte_len, input_size, row_count, 0, out_handle);
}

int hpc_weight_upload_device(int type_id, const void* d_bytes, size_t byte_len, size_t input_size, size_t row_count,
                             void* stream, hpc_weight* out_handle) {
  return upload_common(type_id, d_bytes, true, byte_len, input_size, row_count, static_cast<cudaStream_t>(stream),
                       out_handle);
}

int hpc_weight_release(hpc_weight h) {
  if (!valid(h)) return fail(HPC_ERR_ARG, "invalid weight handle");
  cudaError_t e = cudaFree(h->d_data);
  h->magic = 0;
  h->d_data = nullptr;
  delete h;
  if (e != cudaSuccess) return cuda_fail(e, "cudaFree(weight)");
  return HPC_OK;
}

int hpc_weight_info(hpc_weight h, int* type_id, size_t* input_size, size_t* row_count, size_t* device_bytes) {
  if (!valid(h)) return fail(HPC_ERR_ARG, "invalid weight handle");
  if (type_id) *type_id = h->type;
  if (input_size) *input_size = h->input_size;
  if (row_count) *row_count = h->row_count;
  if (device_bytes) *device_bytes = h->bytes;
  return HPC_OK;
}

int hpc_weight_dequantize(hpc_weight h, float* d_out, size_t out_len, void* stream) {
  if (!valid(h)) return fail(HPC_ERR_ARG, "invalid weight handle");
  if (out_len != h->input_size * h->row_count) return fail(HPC_ERR_SHAPE, "dequantize output length %zu", out_len);
  if (!d_out) return fail(HPC_ERR_ARG, "null output");
  HPC_CK(hc::launch_dequant(h->type, h->d_data, d_out, int(h->row_count), h->nb, static_cast<cudaStream_t>(stream)),
         "dequantize launch");
  return HPC_OK;
}

int hpc_quantize_q8_k(const float* d_in, size_t in_len, size_t input_size, size_t column_count, float* d_d,
                      int8_t* d_qs, int16_t* d_bsums, void* stream) {
  if (input_size == 0 || input_size % 256 || in_len != input_size * column_count)
    return fail(HPC_ERR_SHAPE, "quantize_q8_k shape mismatch");
  if (column_count == 0) return HPC_OK;
  if (!d_in || !d_d || !d_qs || !d_bsums) return fail(HPC_ERR_ARG, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int K = int(input_size), cols = int(column_count);
  void* ws = nullptr;
  HPC_CK(cudaMallocAsync(&ws, hc::q8buf_bytes(K, cols), st), "cudaMallocAsync(q8)");
  hc::Q8Buf q = hc::q8buf_carve(ws, K, cols);
  cudaError_t e = hc::launch_q8k_quantize(d_in, K, cols, q, d_qs, d_bsums, d_d, st);
  cudaFreeAsync(ws, st);
  if (e != cudaSuccess) return cuda_fail(e, "quantize_q8_k launch");
  return HPC_OK;
}

// Narrowest launch (columns) that runs on the tensor-core GEMV:
// GEMV_MMA_MIN_COLS, or HPC_GEMV_MMA_MIN_COLS (9 keeps every launch of up to
// 8 columns on the dp4a GEMV).
static int gemv_mma_min_cols() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("HPC_GEMV_MMA_MIN_COLS");
    v = e ? atoi(e) : hc::GEMV_MMA_MIN_COLS;
    if (v < 1) v = 1;
  }
  return v;
}

// Exact-order launches (hc_gemvx.cu): one per group of up to 8 columns.
static int launch_gemvx_ws(const hc::Q8Buf& q, int K, int cols, const hc::GemvSeg* segs, int nseg, int total_tiles,
                           cudaStream_t st, const hc::GemvPrologue* pro = nullptr) {
  hc::GemvxParams p;
  memset(&p, 0, sizeof p);
  if (pro) p.pro = *pro;
  for (int i = 0; i < nseg; ++i) p.seg[i] = segs[i];
  p.nseg = nseg;
  p.K = K;
  p.nb = K / 256;
  p.total_tiles = total_tiles;
  p.q = q;
  // widest column groups the warp-per-tile form takes, or whose products fit
  // a CTA's shared memory in the split form
  int group = hc::GEMVX_MAX_COLS;
  for (; group > 1; group >>= 1) {
    hc::GemvxParams t = p;
    t.ncols = cols < group ? cols : group;
    int wgrid = 0;
    if (hc::gemvw_plan(t, hc::sm_count(), &wgrid) > 0 && wgrid > 0) break;
    t = p;
    t.ncols = cols < group ? cols : group;
    if (hc::gemvx_plan(t, hc::sm_count()) > 0) break;
  }
  for (int c0 = 0; c0 < cols; c0 += group) {
    p.col0 = c0;
    p.ncols = cols - c0 < group ? cols - c0 : group;
    HPC_CK(hc::launch_gemvx(p, st), "exact-order gemv launch");
  }
  return HPC_OK;
}

// GEMV launches over an already-quantized workspace.  Fewer than TC_MIN_COLS
// columns: `exact` selects the reference-order kernel (hc_gemvx.cu), else the
// dp4a GEMV (1-2 columns per launch, optionally with the fused norm prologue)
// or the tensor-core GEMV (3-8), one launch per group of up to 8 columns
// covering all segments.  TC_MIN_COLS or more: the tensor-core matmul.
static int launch_gemv_ws(const hc::Q8Buf& q, int K, int cols, const hc::GemvSeg* segs, int nseg, int total_tiles,
                          cudaStream_t st, const hc::GemvPrologue* pro, bool exact) {
  if (exact && !pro && cols < hc::TC_MIN_COLS) return launch_gemvx_ws(q, K, cols, segs, nseg, total_tiles, st);
  hc::GemvParams p;
  memset(&p, 0, sizeof p);
  if (pro) p.pro = *pro;
  for (int i = 0; i < nseg; ++i) p.seg[i] = segs[i];
  p.nseg = nseg;
  p.K = K;
  p.nb = K / 256;
  p.total_tiles = total_tiles;
  p.q = q;
  if (cols >= hc::TC_MIN_COLS && !pro) {
    for (int i = 0; i < nseg; ++i) HPC_CK(hc::launch_gemm_tc(segs[i], K / 256, q, 0, cols, st), "tensor-core matmul");
    return HPC_OK;
  }
  for (int c0 = 0; c0 < cols; c0 += 8) {
    p.col0 = c0;
    p.ncols = cols - c0 < 8 ? cols - c0 : 8;
    if (p.ncols >= gemv_mma_min_cols() && !pro) {
      HPC_CK(hc::launch_gemv_mma(p, st), "tensor-core gemv launch");
      continue;
    }
    hc::gemv_plan(p);  // the plan depends on the column count of the launch
    HPC_CK(hc::launch_gemv(p, st), "gemv launch");
  }
  return HPC_OK;
}

// Shared by the single and multi entry points: quantize once into a
// stream-ordered scratch allocation, then the GEMV launches.
static int run_gemv(const float* d_in, int K, int cols, const hc::GemvSeg* segs, int nseg, int total_tiles,
                    cudaStream_t st) {
  if (cols == 0) return HPC_OK;
  void* ws = nullptr;
  HPC_CK(cudaMallocAsync(&ws, hc::q8buf_bytes(K, cols), st), "cudaMallocAsync(q8)");
  hc::Q8Buf q = hc::q8buf_carve(ws, K, cols);
  cudaError_t e = hc::launch_q8k_quantize(d_in, K, cols, q, nullptr, nullptr, nullptr, st);
  int rc = e == cudaSuccess ? launch_gemv_ws(q, K, cols, segs, nseg, total_tiles, st, nullptr, g_exact_order.load())
                            : cuda_fail(e, "quantize launch");
  cudaError_t e2 = cudaFreeAsync(ws, st);
  if (rc != HPC_OK) return rc;
  if (e2 != cudaSuccess) return cuda_fail(e2, "cudaFreeAsync(q8)");
  return HPC_OK;
}

// Validates `count` handles against (input_size, column_count) and fills the
// segment table; returns the total tile count through *tiles.
static int build_segments(size_t count, const hpc_weight* handles, float* const* d_outs, const size_t* out_lens,
                          size_t input_size, size_t column_count, hc::GemvSeg* segs, int* tiles_out) {
  int dev = 0;
  HPC_CK(cudaGetDevice(&dev), "cudaGetDevice");
  int tiles = 0;
  for (size_t i = 0; i < count; ++i) {
    const hpc_weight h = handles[i];
    if (!valid(h)) return fail(HPC_ERR_ARG, "invalid weight handle %zu", i);
    size_t rb;
    if (!row_bytes(h->type, input_size, &rb)) return fail(HPC_ERR_TYPE, "unsupported type %d", h->type);
    if (h->input_size != input_size || out_lens[i] != h->row_count * column_count)
      return fail(HPC_ERR_SHAPE, "matmul: spec %zu shape mismatch", i);
    if (h->device != dev) return fail(HPC_ERR_ARG, "handle %zu lives on device %d, current device is %d", i, h->device, dev);
    if (column_count > 0 && !d_outs[i]) return fail(HPC_ERR_ARG, "null output %zu", i);
    segs[i].w = h->d_data;
    segs[i].out = d_outs[i];
    segs[i].type = h->type;
    segs[i].rows = int(h->row_count);
    segs[i].tile_begin = tiles;
    segs[i].pad = 0;
    tiles += int(h->rows_pad / hc::TILE);
  }
  *tiles_out = tiles;
  return HPC_OK;
}

int hpc_matmul_quantized_prepared_f32(hpc_weight h, const float* d_in, size_t in_len, size_t input_size,
                                      size_t row_count, size_t column_count, float* d_out, size_t out_len,
                                      void* stream) {
  if (in_len != input_size * column_count || out_len != row_count * column_count)
    return fail(HPC_ERR_SHAPE, "matmul shape mismatch: input %zu output %zu", in_len, out_len);
  if (!valid(h)) return fail(HPC_ERR_ARG, "invalid weight handle");
  size_t rb;
  if (!row_bytes(h->type, input_size, &rb)) return fail(HPC_ERR_TYPE, "unsupported type %d for input size %zu", h->type, input_size);
  if (h->input_size != input_size || h->row_count != row_count)
    return fail(HPC_ERR_SHAPE, "handle shape mismatch: %zux%zu vs %zux%zu", h->input_size, h->row_count, input_size, row_count);
  if (column_count > 0 && (!d_in || !d_out)) return fail(HPC_ERR_ARG, "null pointer");
  if (column_count > (size_t(1) << 20)) return fail(HPC_ERR_SHAPE, "too many columns");
  hc::GemvSeg s;
  int tiles = 0;
  int rc = build_segments(1, &h, &d_out, &out_len, input_size, column_count, &s, &tiles);
  if (rc != HPC_OK) return rc;
  return run_gemv(d_in, int(input_size), int(column_count), &s, 1, tiles, static_cast<cudaStream_t>(stream));
}

int hpc_matmul_quantized_prepared_multi_f32(size_t count, const float* d_in, size_t in_len, size_t input_size,
                                            size_t column_count, const hpc_weight* handles, float* const* d_outs,
                                            const size_t* out_lens, void* stream) {
  if (count == 0 || count > size_t(hc::GEMV_MAXSEG) || in_len != input_size * column_count)
    return fail(HPC_ERR_SHAPE, "multi matmul: count %zu / input length %zu", count, in_len);
  if (!handles || !d_outs || !out_lens) return fail(HPC_ERR_ARG, "null pointer");
  if (column_count > (size_t(1) << 20)) return fail(HPC_ERR_SHAPE, "too many columns");
  hc::GemvSeg segs[hc::GEMV_MAXSEG];
  int tiles = 0;
  int rc = build_segments(count, handles, d_outs, out_lens, input_size, column_count, segs, &tiles);
  if (rc != HPC_OK) return rc;
  if (column_count > 0 && !d_in) return fail(HPC_ERR_ARG, "null input");
  return run_gemv(d_in, int(input_size), int(column_count), segs, int(count), tiles, static_cast<cudaStream_t>(stream));
}

int hpc_matmul_quantized_f32(int type_id, const uint8_t* host_weight, size_t weight_len, const float* host_in,
                             size_t in_len, size_t input_size, size_t row_count, size_t column_count, float* host_out,
                             size_t out_len) {
  if (in_len != input_size * column_count || out_len != row_count * column_count)
    return fail(HPC_ERR_SHAPE, "matmul shape mismatch");
  size_t rb;
  if (!row_bytes(type_id, input_size, &rb)) return fail(HPC_ERR_TYPE, "unsupported type %d", type_id);
  if (weight_len != rb * row_count) return fail(HPC_ERR_SHAPE, "weight length %zu", weight_len);
  if (column_count == 0 || row_count == 0) return HPC_OK;
  if (!host_in || !host_out) return fail(HPC_ERR_ARG, "null pointer");
  hpc_weight h = nullptr;
  int rc = hpc_weight_upload(type_id, host_weight, weight_len, input_size, row_count, &h);
  if (rc != HPC_OK) return rc;
  float* d_in = nullptr;
  float* d_out = nullptr;
  cudaError_t e = cudaMalloc(&d_in, in_len * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&d_out, out_len * sizeof(float));
  if (e == cudaSuccess) e = cudaMemcpy(d_in, host_in, in_len * sizeof(float), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    rc = hpc_matmul_quantized_prepared_f32(h, d_in, in_len, input_size, row_count, column_count, d_out, out_len, nullptr);
    if (rc == HPC_OK) e = cudaMemcpy(host_out, d_out, out_len * sizeof(float), cudaMemcpyDeviceToHost);
  }
  cudaFree(d_in);
  cudaFree(d_out);
  hpc_weight_release(h);
  if (rc != HPC_OK) return rc;
  if (e != cudaSuccess) return cuda_fail(e, "one-shot matmul");
  return HPC_OK;
}

int hpc_matmul_dequantized_prepared_f32(hpc_weight h, const float* d_in, size_t in_len, size_t input_size,
                                        size_t row_count, size_t column_count, float* d_out, size_t out_len,
                                        void* stream) {
  if (in_len != input_size * column_count || out_len != row_count * column_count)
    return fail(HPC_ERR_SHAPE, "dequantized matmul shape mismatch: input %zu output %zu", in_len, out_len);
  if (!valid(h)) return fail(HPC_ERR_ARG, "invalid weight handle");
  size_t rb;
  if (!row_bytes(h->type, input_size, &rb)) return fail(HPC_ERR_TYPE, "unsupported type %d for input size %zu", h->type, input_size);
  if (h->input_size != input_size || h->row_count != row_count)
    return fail(HPC_ERR_SHAPE, "handle shape mismatch: %zux%zu vs %zux%zu", h->input_size, h->row_count, input_size, row_count);
  if (column_count == 0 || row_count == 0) return HPC_OK;
  if (!d_in || !d_out) return fail(HPC_ERR_ARG, "null pointer");
  if (column_count > size_t(65535) * 8) return fail(HPC_ERR_SHAPE, "too many columns");
  int dev = 0;
  HPC_CK(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != h->device) return fail(HPC_ERR_ARG, "weight on device %d, current %d", h->device, dev);
  HPC_CK(hc::launch_dequant_matmul(h->type, h->d_data, h->nb, int(row_count), int(h->rows_pad), d_in, int(input_size),
                                   int(column_count), d_out, static_cast<cudaStream_t>(stream)),
         "dequantized matmul launch");
  return HPC_OK;
}

int hpc_matmul_dequantized_f32(int type_id, const uint8_t* host_weight, size_t weight_len, const float* host_in,
                               size_t in_len, size_t input_size, size_t row_count, size_t column_count, float* host_out,
                               size_t out_len) {
  if (in_len != input_size * column_count || out_len != row_count * column_count)
    return fail(HPC_ERR_SHAPE, "dequantized matmul shape mismatch");
  size_t rb;
  if (!row_bytes(type_id, input_size, &rb)) return fail(HPC_ERR_TYPE, "unsupported type %d", type_id);
  if (weight_len != rb * row_count) return fail(HPC_ERR_SHAPE, "weight length %zu", weight_len);
  if (column_count == 0 || row_count == 0) return HPC_OK;
  if (!host_in || !host_out) return fail(HPC_ERR_ARG, "null pointer");
  hpc_weight h = nullptr;
  int rc = hpc_weight_upload(type_id, host_weight, weight_len, input_size, row_count, &h);
  if (rc != HPC_OK) return rc;
  float* d_in = nullptr;
  float* d_out = nullptr;
  cudaError_t e = cudaMalloc(&d_in, in_len * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&d_out, out_len * sizeof(float));
  if (e == cudaSuccess) e = cudaMemcpy(d_in, host_in, in_len * sizeof(float), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    rc = hpc_matmul_dequantized_prepared_f32(h, d_in, in_len, input_size, row_count, column_count, d_out, out_len,
                                             nullptr);
    if (rc == HPC_OK) e = cudaMemcpy(host_out, d_out, out_len * sizeof(float), cudaMemcpyDeviceToHost);
  }
  cudaFree(d_in);
  cudaFree(d_out);
  hpc_weight_release(h);
  if (rc != HPC_OK) return rc;
  if (e != cudaSuccess) return cuda_fail(e, "one-shot dequantized matmul");
  return HPC_OK;
}

int hpc_q8_workspace_bytes(size_t input_size, size_t column_count, size_t* out_bytes) {
  if (!out_bytes) return fail(HPC_ERR_ARG, "null out_bytes");
  if (input_size == 0 || input_size % 256 || column_count > (size_t(1) << 20))
    return fail(HPC_ERR_SHAPE, "workspace shape %zu x %zu", input_size, column_count);
  *out_bytes = hc::q8buf_bytes(int(input_size), int(column_count));
  return HPC_OK;
}

int hpc_q8_quantize(const float* d_in, size_t in_len, size_t input_size, size_t column_count, void* d_workspace,
                    size_t workspace_bytes, void* stream) {
  if (input_size == 0 || input_size % 256 || in_len != input_size * column_count || column_count > (size_t(1) << 20))
    return fail(HPC_ERR_SHAPE, "q8 quantize shape mismatch");
  if (column_count == 0) return HPC_OK;
  if (!d_in || !d_workspace) return fail(HPC_ERR_ARG, "null pointer");
  if (workspace_bytes < hc::q8buf_bytes(int(input_size), int(column_count)))
    return fail(HPC_ERR_SHAPE, "workspace too small: %zu bytes", workspace_bytes);
  hc::Q8Buf q = hc::q8buf_carve(d_workspace, int(input_size), int(column_count));
  HPC_CK(hc::launch_q8k_quantize(d_in, int(input_size), int(column_count), q, nullptr, nullptr, nullptr,
                                 static_cast<cudaStream_t>(stream)), "quantize launch");
  return HPC_OK;
}

int hpc_matmul_q8(size_t count, const hpc_weight* handles, const void* d_workspace, size_t workspace_bytes,
                  size_t input_size, size_t column_count, float* const* d_outs, const size_t* out_lens, void* stream) {
  return hc_matmul_q8_order(count, handles, d_workspace, workspace_bytes, input_size, column_count, d_outs, out_lens,
                            g_exact_order.load(), static_cast<cudaStream_t>(stream));
}

int hpc_set_matmul_order(int exact) {
  g_exact_order.store(exact != 0);
  return HPC_OK;
}

}  // extern "C"

int hc_matmul_q8_order(size_t count, const hpc_weight* handles, const void* d_workspace, size_t workspace_bytes,
                       size_t input_size, size_t column_count, float* const* d_outs, const size_t* out_lens,
                       bool exact, cudaStream_t stream) {
  if (count == 0 || count > size_t(hc::GEMV_MAXSEG)) return fail(HPC_ERR_SHAPE, "matmul_q8: count %zu", count);
  if (!handles || !d_outs || !out_lens) return fail(HPC_ERR_ARG, "null pointer");
  if (input_size == 0 || input_size % 256 || column_count > (size_t(1) << 20))
    return fail(HPC_ERR_SHAPE, "matmul_q8 shape");
  if (column_count > 0 && !d_workspace) return fail(HPC_ERR_ARG, "null workspace");
  if (workspace_bytes < hc::q8buf_bytes(int(input_size), int(column_count)))
    return fail(HPC_ERR_SHAPE, "workspace too small: %zu bytes", workspace_bytes);
  hc::GemvSeg segs[hc::GEMV_MAXSEG];
  int tiles = 0;
  int rc = build_segments(count, handles, d_outs, out_lens, input_size, column_count, segs, &tiles);
  if (rc != HPC_OK) return rc;
  if (column_count == 0) return HPC_OK;
  hc::Q8Buf q = hc::q8buf_carve(const_cast<void*>(d_workspace), int(input_size), int(column_count));
  return launch_gemv_ws(q, int(input_size), int(column_count), segs, int(count), tiles, stream, nullptr, exact);
}

// The exact-order matmul whose input every CTA computes itself
// (GemvPrologue: the norms of the residual stream, or the Q8_K of a
// vector as it is): the exact decode step's QKV, O and gate/up projections
// of width 2048, any column count up to the model's step width.
int hc_matmul_q8_exact_prologue(size_t count, const hpc_weight* handles, const void* q8ws, size_t q8_bytes,
                                size_t input_size, size_t column_count, float* const* d_outs, const size_t* out_lens,
                                const hc::GemvPrologue& pro, cudaStream_t st) {
  if (count == 0 || count > size_t(hc::GEMV_MAXSEG)) return fail(HPC_ERR_SHAPE, "matmul_q8: count %zu", count);
  if (input_size != size_t(hc::GEMV_PRO_D) || column_count < 1 || column_count > size_t(hc::GEMVX_MAX_COLS))
    return fail(HPC_ERR_SHAPE, "exact prologue: width %zu, %zu columns", input_size, column_count);
  if (q8_bytes < hc::q8buf_bytes(int(input_size), int(column_count))) return fail(HPC_ERR_SHAPE, "workspace too small");
  hc::GemvSeg segs[hc::GEMV_MAXSEG];
  int tiles = 0;
  int rc = build_segments(count, handles, d_outs, out_lens, input_size, column_count, segs, &tiles);
  if (rc != HPC_OK) return rc;
  hc::Q8Buf q = hc::q8buf_carve(const_cast<void*>(q8ws), int(input_size), int(column_count));
  return launch_gemvx_ws(q, int(input_size), int(column_count), segs, int(count), tiles, st, &pro);
}

// hpc_matmul_q8 whose input is computed by the fused norm prologue of every
// CTA (hc_kernels.cuh GemvPrologue) instead of read from Q8_K records: the
// decode step's QKV and gate/up projections for one or two columns of width
// 2048.  `q8ws` still carries the record geometry of the launch.
int hc_matmul_q8_prologue(size_t count, const hpc_weight* handles, const void* q8ws, size_t q8_bytes, size_t input_size,
                          size_t column_count, float* const* d_outs, const size_t* out_lens,
                          const hc::GemvPrologue& pro, cudaStream_t st) {
  if (count == 0 || count > size_t(hc::GEMV_MAXSEG)) return fail(HPC_ERR_SHAPE, "matmul_q8: count %zu", count);
  if (input_size != size_t(hc::GEMV_PRO_D) || column_count < 1 || column_count > 2)
    return fail(HPC_ERR_SHAPE, "fused prologue: width %zu, %zu columns", input_size, column_count);
  if (q8_bytes < hc::q8buf_bytes(int(input_size), int(column_count))) return fail(HPC_ERR_SHAPE, "workspace too small");
  hc::GemvSeg segs[hc::GEMV_MAXSEG];
  int tiles = 0;
  int rc = build_segments(count, handles, d_outs, out_lens, input_size, column_count, segs, &tiles);
  if (rc != HPC_OK) return rc;
  hc::Q8Buf q = hc::q8buf_carve(const_cast<void*>(q8ws), int(input_size), int(column_count));
  return launch_gemv_ws(q, int(input_size), int(column_count), segs, int(count), tiles, st, &pro, false);
}

extern "C" {

int hpc_set_wide_matmul_kind(int kind) {
  if (kind != 0 && kind != 1) return fail(HPC_ERR_ARG, "wide matmul kind %d", kind);
  hc::set_gemm_t5(kind == 1);
  return HPC_OK;
}

int hpc_matmul_rmsnorm_f32(size_t count, const hpc_weight* handles, void* d_workspace, size_t workspace_bytes,
                           size_t input_size, size_t column_count, const float* d_x, const float* d_y,
                           const float* d_w_post, const float* d_w_pre, double eps, float* d_x_out,
                           float* const* d_outs, const size_t* out_lens, void* stream) {
  if (!handles || !d_workspace || !d_x || !d_w_pre || !d_outs || !out_lens) return fail(HPC_ERR_ARG, "null pointer");
  if (d_y && (!d_w_post || !d_x_out)) return fail(HPC_ERR_ARG, "residual form needs w_post and x_out");
  if (d_y && d_x_out == d_x) return fail(HPC_ERR_ARG, "x_out aliases x");
  hc::GemvPrologue pro{};
  pro.mode = d_y ? hc::GEMV_PRO_RESID_NORM : hc::GEMV_PRO_NORM;
  pro.x = d_x;
  pro.y = d_y;
  pro.w_post = d_w_post;
  pro.w_pre = d_w_pre;
  pro.x_out = d_x_out;
  pro.eps = eps;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (g_exact_order.load())
    return hc_matmul_q8_exact_prologue(count, handles, d_workspace, workspace_bytes, input_size, column_count, d_outs,
                                       out_lens, pro, st);
  return hc_matmul_q8_prologue(count, handles, d_workspace, workspace_bytes, input_size, column_count, d_outs,
                               out_lens, pro, st);
}

}  // extern "C"

extern "C" {

static int lm_head_check(hpc_weight h, size_t input_size, size_t column_count, size_t k) {
  if (!valid(h)) return fail(HPC_ERR_ARG, "invalid weight handle");
  if (h->input_size != input_size) return fail(HPC_ERR_SHAPE, "LM head input size %zu vs %zu", h->input_size, input_size);
  if (k < 1 || k > size_t(hc::TOPK_MAX) || k > h->row_count)
    return fail(HPC_ERR_SHAPE, "top-k %zu outside 1..min(64, rows)", k);
  if (column_count > (size_t(1) << 20)) return fail(HPC_ERR_SHAPE, "too many columns");
  int dev = 0;
  HPC_CK(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev != h->device) return fail(HPC_ERR_ARG, "handle lives on device %d, current device is %d", h->device, dev);
  return HPC_OK;
}

// Inputs of >= TC_MIN_COLS columns take the tensor-core path: the logits
// [col][rows] (256-byte aligned) followed by one candidate list per
// LOGITS_CHUNK_ROWS-row chunk per column.  Narrower inputs: one list per CTA
// of the fused GEMV + top-k kernel.
static size_t tc_chunks(hpc_weight h) { return (h->row_count + hc::LOGITS_CHUNK_ROWS - 1) / hc::LOGITS_CHUNK_ROWS; }
static size_t tc_logits_bytes(hpc_weight h, size_t cols) { return (cols * h->row_count * sizeof(float) + 255) / 256 * 256; }

// Inputs of GEMV_MMA_MIN_COLS .. 8 columns: the tensor-core LM head + top-k,
// one list per CTA of its persistent grid.
static bool lm_head_mma(size_t cols) { return cols >= size_t(gemv_mma_min_cols()) && cols <= 8; }

// Logits path (tensor-core matmul at TC_MIN_COLS+ columns, the exact-order
// GEMV at 3..TC_MIN_COLS-1): the logits [col][rows] (256-byte aligned), then
// one candidate list per 2,048-row chunk and column.
static size_t logits_path_bytes(hpc_weight h, size_t cols, size_t k) {
  return tc_logits_bytes(h, cols) + tc_chunks(h) * k * cols * sizeof(uint64_t);
}

// Candidate bytes for `cols` columns: enough for every path the width may
// take in either order (the model's reordered step and the exact one share
// one buffer).
static size_t cand_bytes_for(hpc_weight h, size_t cols, size_t k) {
  if (cols >= size_t(hc::TC_MIN_COLS)) return logits_path_bytes(h, cols, k);
  const int tiles = int(h->rows_pad / hc::TILE);
  size_t b = size_t(hc::lmhead_grid(tiles)) * hc::LMHEAD_LISTS * k * cols * sizeof(uint64_t);
  if (lm_head_mma(cols)) b = std::max(b, size_t(hc::lmhead_mma_grid(tiles)) * k * cols * sizeof(uint64_t));
  if (cols >= 3) b = std::max(b, logits_path_bytes(h, cols, k));
  return b;
}

int hpc_lm_head_candidates_bytes(hpc_weight h, size_t column_count, size_t k, size_t* out_bytes) {
  if (!out_bytes) return fail(HPC_ERR_ARG, "null out_bytes");
  int rc = lm_head_check(h, h ? h->input_size : 0, column_count, k);
  if (rc != HPC_OK) return rc;
  *out_bytes = cand_bytes_for(h, column_count, k);
  return HPC_OK;
}

int hpc_lm_head_topk_q8(hpc_weight h, const void* d_workspace, size_t workspace_bytes, size_t input_size,
                        size_t column_count, size_t k, int32_t id_offset, void* d_candidates, size_t candidates_bytes,
                        float softcap, int32_t* d_ids, float* d_vals, uint64_t* d_keys, void* stream) {
  return hc_lm_head_topk_q8_order(h, d_workspace, workspace_bytes, input_size, column_count, k, id_offset,
                                  d_candidates, candidates_bytes, softcap, d_ids, d_vals, d_keys, g_exact_order.load(),
                                  static_cast<cudaStream_t>(stream));
}

}  // extern "C"

size_t hc_lm_head_fused_candidates_bytes(hpc_weight h, size_t cols, size_t k) {
  return size_t(hc::lmhead_grid(int(h->rows_pad / hc::TILE))) * hc::LMHEAD_LISTS * k * cols * sizeof(uint64_t);
}

int hc_lm_head_topk_q8_order(hpc_weight h, const void* d_workspace, size_t workspace_bytes, size_t input_size,
                             size_t column_count, size_t k, int32_t id_offset, void* d_candidates,
                             size_t candidates_bytes, float softcap, int32_t* d_ids, float* d_vals, uint64_t* d_keys,
                             bool exact, cudaStream_t st, bool fused_only) {
  int rc = lm_head_check(h, input_size, column_count, k);
  if (rc != HPC_OK) return rc;
  if (column_count == 0) return HPC_OK;
  if (!d_workspace || !d_candidates || !d_ids || !d_vals) return fail(HPC_ERR_ARG, "null pointer");
  if (workspace_bytes < hc::q8buf_bytes(int(input_size), int(column_count)))
    return fail(HPC_ERR_SHAPE, "workspace too small: %zu bytes", workspace_bytes);
  const size_t need = fused_only ? hc_lm_head_fused_candidates_bytes(h, column_count, k)
                                 : cand_bytes_for(h, column_count, k);
  if (candidates_bytes < need) return fail(HPC_ERR_SHAPE, "candidate buffer too small: %zu bytes", candidates_bytes);
  if (id_offset < 0 || size_t(id_offset) + h->row_count > size_t(INT32_MAX)) return fail(HPC_ERR_SHAPE, "id offset");
  if (fused_only) exact = true;
  if (!fused_only && (column_count >= size_t(hc::TC_MIN_COLS) || (exact && column_count >= 3))) {
    // the logits (tensor-core matmul, or the exact-order GEMV), chunked
    // candidate lists, then the same merge
    float* logits = static_cast<float*>(d_candidates);
    uint64_t* cand = reinterpret_cast<uint64_t*>(static_cast<char*>(d_candidates) + tc_logits_bytes(h, column_count));
    hc::GemvSeg seg;
    memset(&seg, 0, sizeof seg);
    seg.w = h->d_data;
    seg.out = logits;
    seg.type = h->type;
    seg.rows = int(h->row_count);
    seg.tile_begin = 0;
    const hc::Q8Buf q = hc::q8buf_carve(const_cast<void*>(d_workspace), int(input_size), int(column_count));
    if (column_count >= size_t(hc::TC_MIN_COLS)) {
      HPC_CK(hc::launch_gemm_tc(seg, int(input_size / 256), q, 0, int(column_count), st), "tensor-core LM head");
    } else {
      rc = launch_gemvx_ws(q, int(input_size), int(column_count), &seg, 1, int(h->rows_pad / hc::TILE), st);
      if (rc != HPC_OK) return rc;
    }
    const size_t col_stride = tc_chunks(h) * k;
    HPC_CK(hc::launch_logits_topk(logits, int(h->row_count), int(column_count), int(k), id_offset, cand, col_stride,
                                  st),
           "logits top-k");
    HPC_CK(hc::launch_topk_merge(cand, int(col_stride), col_stride, int(k), k, int(column_count), int(k), softcap,
                                 d_ids, d_vals, d_keys, st),
           "top-k merge launch");
    return HPC_OK;
  }
  const int tiles = int(h->rows_pad / hc::TILE);
  const int grid = hc::lmhead_grid(tiles);
  hc::LmHeadParams P;
  memset(&P, 0, sizeof P);
  P.g.seg[0].w = h->d_data;
  P.g.seg[0].out = nullptr;
  P.g.seg[0].type = h->type;
  P.g.seg[0].rows = int(h->row_count);
  P.g.nseg = 1;
  P.g.K = int(input_size);
  P.g.nb = int(input_size / 256);
  P.g.split = 1;
  P.g.split_log2 = 0;
  P.g.bps = P.g.nb;
  P.g.bulk = 0;
  P.g.err = hc::device_status_word();
  P.g.total_tiles = tiles;
  P.g.q = hc::q8buf_carve(const_cast<void*>(d_workspace), int(input_size), int(column_count));
  P.k = int(k);
  P.id_offset = id_offset;
  P.cand = static_cast<uint64_t*>(d_candidates);
  const int cols = int(column_count);
  if (!exact && !fused_only && lm_head_mma(column_count)) {
    const int mgrid = hc::lmhead_mma_grid(tiles);
    P.cand_col_stride = size_t(mgrid) * k;
    P.g.col0 = 0;
    P.g.ncols = cols;
    HPC_CK(hc::launch_lmhead_mma(P, mgrid, st), "tensor-core lm head launch");
    HPC_CK(hc::launch_topk_merge(P.cand, mgrid * int(k), P.cand_col_stride, int(k), k, cols, int(k), softcap, d_ids,
                                 d_vals, d_keys, st),
           "top-k merge launch");
    return HPC_OK;
  }
  P.cand_col_stride = size_t(grid) * hc::LMHEAD_LISTS * k;
  // exact order: passes of at most 2 columns (the kernel's exact lane
  // accumulators of wider passes would not fit its registers)
  const int group = exact ? 2 : 8;
  for (int c0 = 0; c0 < cols; c0 += group) {
    P.g.col0 = c0;
    P.g.ncols = cols - c0 < group ? cols - c0 : group;
    HPC_CK(hc::launch_lmhead_topk(P, grid, st), "lm head launch");
  }
  const int n = grid * hc::LMHEAD_LISTS * int(k);
  HPC_CK(hc::launch_topk_merge(P.cand, n, P.cand_col_stride, int(k), k, cols, int(k), softcap, d_ids, d_vals, d_keys,
                               st),
         "top-k merge launch");
  return HPC_OK;
}

extern "C" {

int hpc_lm_head_topk(hpc_weight h, const float* d_hidden, size_t hidden_len, size_t input_size, size_t column_count,
                     size_t k, int32_t id_offset, float softcap, int32_t* d_ids, float* d_vals, void* stream) {
  if (hidden_len != input_size * column_count) return fail(HPC_ERR_SHAPE, "hidden length %zu", hidden_len);
  int rc = lm_head_check(h, input_size, column_count, k);
  if (rc != HPC_OK) return rc;
  if (column_count == 0) return HPC_OK;
  if (!d_hidden || !d_ids || !d_vals) return fail(HPC_ERR_ARG, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t qb = hc::q8buf_bytes(int(input_size), int(column_count));
  const size_t cb = cand_bytes_for(h, column_count, k);
  void* ws = nullptr;
  HPC_CK(cudaMallocAsync(&ws, qb + cb, st), "cudaMallocAsync(lm head scratch)");
  hc::Q8Buf q = hc::q8buf_carve(ws, int(input_size), int(column_count));
  cudaError_t e = hc::launch_q8k_quantize(d_hidden, int(input_size), int(column_count), q, nullptr, nullptr, nullptr, st);
  rc = e == cudaSuccess ? hpc_lm_head_topk_q8(h, ws, qb, input_size, column_count, k, id_offset,
                                              static_cast<char*>(ws) + qb, cb, softcap, d_ids, d_vals, nullptr, stream)
                        : cuda_fail(e, "quantize launch");
  cudaError_t e2 = cudaFreeAsync(ws, st);
  if (rc != HPC_OK) return rc;
  if (e2 != cudaSuccess) return cuda_fail(e2, "cudaFreeAsync(lm head scratch)");
  return HPC_OK;
}

int hpc_topk_merge_keys(const uint64_t* d_keys, size_t group_count, size_t column_count, size_t k, float softcap,
                        int32_t* d_ids, float* d_vals, void* stream) {
  if (k < 1 || k > size_t(hc::TOPK_MAX) || group_count == 0 || group_count > 4096 || column_count > (size_t(1) << 20))
    return fail(HPC_ERR_SHAPE, "merge shape: groups %zu columns %zu k %zu", group_count, column_count, k);
  if (column_count == 0) return HPC_OK;
  if (!d_keys || !d_ids || !d_vals) return fail(HPC_ERR_ARG, "null pointer");
  const int n = int(group_count * k);
  HPC_CK(hc::launch_topk_merge(d_keys, n, k, int(k), column_count * k, int(column_count), int(k), softcap, d_ids,
                               d_vals, nullptr, static_cast<cudaStream_t>(stream)),
         "top-k merge launch");
  return HPC_OK;
}

}  // extern "C"
