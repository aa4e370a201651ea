"""Host-side mirror of the reference's kernel bindings, backed by CUDA.

The reference binds its Rust/WASM kernels in
packages/engine/src/runner/wasm/wasm-kernels.ts; this module offers the same
operations with the same argument meaning and the same error behaviour
(assertWasmOk, wasm-kernels.ts:1882-1896 -> assert_cuda_ok), but every call
runs on the GPU through libheliocuda.so:

    reference (wasm-kernels.ts)             here
    ------------------------------------    ---------------------------------------
    matMulQuantizedWasm           :416      mat_mul_quantized
    createWasmQuantizedWeightHandle :520    create_quantized_weight_handle
    releaseWasmQuantizedWeightHandle :576   release_quantized_weight_handle
    matMulQuantizedWasmResident   :593      mat_mul_quantized_resident
    matMulQuantizedWasmResidentMulti :648   mat_mul_quantized_resident_multi
    matMulDequantizedWasm         :468      mat_mul_dequantized
    quantizedTypeId               :1908     quantized_type_id

Activations and outputs are torch CUDA tensors (float32); numpy arrays are
accepted too and are copied to the device and back (the host round trip is
then part of the call, as it is for the WASM linear-memory copies).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib

OK, ERR_SHAPE, ERR_HEADS, ERR_TYPE, ERR_CUDA, ERR_TIMEOUT, ERR_NCCL, ERR_ARG = range(8)

_TYPE_IDS = {"Q4_K": 1, "Q5_K": 2, "Q6_K": 3, "IQ4_XS": 4, "Q8_0": 5, "Q4_0": 6}
_TYPE_NAMES = {v: k for k, v in _TYPE_IDS.items()}


class CudaKernelError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def quantized_type_id(type_name: str) -> int:
    """wasm-kernels.ts:1908-1923."""
    try:
        return _TYPE_IDS[type_name]
    except KeyError:
        raise CudaKernelError(ERR_TYPE, f"unsupported quantized type {type_name}") from None


def assert_cuda_ok(code: int, kernel_name: str) -> None:
    """wasm-kernels.ts:1882-1896, with the GPU codes added."""
    if code == OK:
        return
    detail = _lib.last_error()
    if code == ERR_SHAPE:
        raise CudaKernelError(code, f"{kernel_name} cuda shape mismatch ({detail})")
    if code == ERR_HEADS:
        raise CudaKernelError(code, f"{kernel_name} cuda head count mismatch ({detail})")
    if code == ERR_TYPE:
        raise CudaKernelError(code, f"{kernel_name} cuda unsupported type ({detail})")
    raise CudaKernelError(code, f"{kernel_name} cuda failed with code {code}: {detail}")


def init_device(device: int | None = None) -> int:
    dev = torch.cuda.current_device() if device is None else int(device)
    torch.cuda.set_device(dev)
    assert_cuda_ok(_lib.lib().hpc_device_init(dev), "deviceInit")
    return dev


def _stream() -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _as_device_f32(x) -> tuple[torch.Tensor, bool]:
    """Returns (contiguous cuda float32 tensor, came_from_host)."""
    if isinstance(x, torch.Tensor):
        if not x.is_cuda:
            return x.to(device="cuda", dtype=torch.float32).contiguous(), True
        if x.dtype != torch.float32:
            raise TypeError("activations must be float32")
        return x.contiguous(), False
    arr = np.ascontiguousarray(x, dtype=np.float32)
    return torch.from_numpy(arr).to("cuda"), True


def _ptr(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


@dataclass
class CudaQuantizedWeightHandle:
    """Resident weight in HBM (wasm-kernels.ts:387-397 WasmQuantizedWeightHandle)."""
    type: str
    row_count: int
    input_size: int
    device: int
    device_bytes: int
    _h: C.c_void_p = field(repr=False)
    released: bool = False

    @property
    def handle(self) -> C.c_void_p:
        if self.released:
            raise CudaKernelError(ERR_ARG, "weight handle already released")
        return self._h


def create_quantized_weight_handle(type_name: str, weight_bytes, input_size: int,
                                   row_count: int) -> CudaQuantizedWeightHandle:
    """Upload + repack once (wasm-kernels.ts:520-574).  weight_bytes: host
    bytes/np.uint8, or a uint8 CUDA tensor already on the device."""
    if input_size <= 0 or row_count <= 0:
        raise CudaKernelError(ERR_SHAPE,
                              f"Resident quantized weight shape mismatch: inputSize={input_size} rowCount={row_count}")
    tid = quantized_type_id(type_name)
    h = C.c_void_p()
    if isinstance(weight_bytes, torch.Tensor) and weight_bytes.is_cuda:
        wb = weight_bytes.contiguous()
        code = _lib.lib().hpc_weight_upload_device(tid, _ptr(wb), wb.numel(), input_size, row_count, _stream(),
                                                    C.byref(h))
    else:
        if isinstance(weight_bytes, torch.Tensor):
            weight_bytes = weight_bytes.numpy()
        wb = np.ascontiguousarray(np.frombuffer(weight_bytes, dtype=np.uint8)
                                  if isinstance(weight_bytes, (bytes, bytearray, memoryview)) else weight_bytes,
                                  dtype=np.uint8)
        code = _lib.lib().hpc_weight_upload(tid, wb.ctypes.data_as(C.c_void_p), wb.size, input_size, row_count,
                                            C.byref(h))
    assert_cuda_ok(code, "createQuantizedWeightHandle")
    nbytes = C.c_size_t()
    _lib.lib().hpc_weight_info(h, None, None, None, C.byref(nbytes))
    return CudaQuantizedWeightHandle(type_name, row_count, input_size, torch.cuda.current_device(), nbytes.value, h)


def release_quantized_weight_handle(handle: CudaQuantizedWeightHandle) -> None:
    """wasm-kernels.ts:576-584."""
    if handle.released:
        return
    assert_cuda_ok(_lib.lib().hpc_weight_release(handle.handle), "releaseQuantizedWeightHandle")
    handle.released = True


def dequantize_resident(handle: CudaQuantizedWeightHandle) -> torch.Tensor:
    """f32 [row_count, input_size], bit-exact to lib.rs dequantize_q4_k/q6_k."""
    out = torch.empty((handle.row_count, handle.input_size), dtype=torch.float32, device="cuda")
    assert_cuda_ok(_lib.lib().hpc_weight_dequantize(handle.handle, _ptr(out), out.numel(), _stream()),
                   "dequantizeResident")
    return out


def quantize_q8_k(x: torch.Tensor, input_size: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Q8_K of each column, bit-exact to lib.rs:1774-1811: (d, qs, bsums32)."""
    x, _ = _as_device_f32(x)
    cols = x.numel() // input_size if input_size else 0
    d = torch.empty(cols * (input_size // 256), dtype=torch.float32, device="cuda")
    qs = torch.empty(cols * input_size, dtype=torch.int8, device="cuda")
    bs = torch.empty(cols * (input_size // 32), dtype=torch.int16, device="cuda")
    assert_cuda_ok(_lib.lib().hpc_quantize_q8_k(_ptr(x), x.numel(), input_size, cols, _ptr(d), _ptr(qs), _ptr(bs),
                                                _stream()), "quantizeQ8K")
    return d, qs, bs


def mat_mul_quantized_resident(handle: CudaQuantizedWeightHandle, input_columns, input_size: int, row_count: int,
                               column_count: int):
    """wasm-kernels.ts:593-646 -> hp_matmul_quantized_prepared_f32 (lib.rs:225)."""
    if handle.input_size != input_size or handle.row_count != row_count:
        raise CudaKernelError(ERR_SHAPE, f"Resident quantized matmul handle shape mismatch: "
                                         f"{handle.input_size}x{handle.row_count}")
    x, from_host = _as_device_f32(input_columns)
    if x.numel() != input_size * column_count:
        raise CudaKernelError(ERR_SHAPE, f"Resident quantized matmul input shape mismatch: {x.numel()}")
    out = torch.empty(row_count * column_count, dtype=torch.float32, device="cuda")
    code = _lib.lib().hpc_matmul_quantized_prepared_f32(handle.handle, _ptr(x), x.numel(), input_size, row_count,
                                                        column_count, _ptr(out), out.numel(), _stream())
    assert_cuda_ok(code, "matMulQuantizedResident")
    return out.cpu().numpy() if from_host else out


def mat_mul_quantized_resident_multi(handles, input_columns, input_size: int, column_count: int):
    """wasm-kernels.ts:648-749 -> hp_matmul_quantized_prepared_multi_f32
    (lib.rs:302); one launch for up to 8 weights (the reference takes 2-4)."""
    handles = list(handles)
    if not 1 <= len(handles) <= 8:
        return None
    for h in handles:
        if h.input_size != input_size:
            raise CudaKernelError(ERR_SHAPE, f"Resident quantized multi matmul handle shape mismatch: {h.input_size}")
    x, from_host = _as_device_f32(input_columns)
    if x.numel() != input_size * column_count:
        raise CudaKernelError(ERR_SHAPE, f"Resident quantized multi matmul input shape mismatch: {x.numel()}")
    outs = [torch.empty(h.row_count * column_count, dtype=torch.float32, device="cuda") for h in handles]
    n = len(handles)
    hs = (C.c_void_p * n)(*[h.handle for h in handles])
    os_ = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
    ls = (C.c_size_t * n)(*[o.numel() for o in outs])
    code = _lib.lib().hpc_matmul_quantized_prepared_multi_f32(n, _ptr(x), x.numel(), input_size, column_count, hs, os_,
                                                              ls, _stream())
    assert_cuda_ok(code, "MatMulQuantizedResidentMulti")
    return [o.cpu().numpy() for o in outs] if from_host else outs


def set_wide_matmul_kind(kind: int) -> None:
    """Tensor-core kind of the >= 16-column Q4_K matmul: 0 = mma.sync
    (default), 1 = tcgen05 (hpc_set_wide_matmul_kind)."""
    assert_cuda_ok(_lib.lib().hpc_set_wide_matmul_kind(int(kind)), "setWideMatmulKind")


def mat_mul_rmsnorm(handles, x, w_pre, column_count: int, *, y=None, w_post=None, eps: float = 1e-6):
    """The decode step's norm-fused projection (hpc_matmul_rmsnorm_f32):
    h = x + rmsNorm(y) * w_post (or x when y is None), then every weight
    times Q8_K(rmsNorm(h) * w_pre) -- wasm/layers.ts:161-247's rmsNorm,
    quantize_q8_k and hp_matmul_quantized_prepared_multi_f32 in one launch.
    Device tensors in; returns (outputs, h or None)."""
    handles = list(handles)
    n = len(handles)
    if not 1 <= n <= 8:
        raise CudaKernelError(ERR_SHAPE, f"matMulRmsNorm: {n} weights")
    d = int(handles[0].input_size)
    for t in (x, w_pre) + ((y, w_post) if y is not None else ()):
        if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
            raise CudaKernelError(ERR_ARG, "matMulRmsNorm: contiguous f32 device tensors")
    nbytes = C.c_size_t()
    assert_cuda_ok(_lib.lib().hpc_q8_workspace_bytes(d, column_count, C.byref(nbytes)), "q8 workspace")
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")
    outs = [torch.empty(h.row_count * column_count, dtype=torch.float32, device="cuda") for h in handles]
    x_out = torch.empty_like(x) if y is not None else None
    hs = (C.c_void_p * n)(*[h.handle for h in handles])
    os_ = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
    ls = (C.c_size_t * n)(*[o.numel() for o in outs])
    code = _lib.lib().hpc_matmul_rmsnorm_f32(n, hs, _ptr(ws), nbytes.value, d, column_count, _ptr(x),
                                             _ptr(y) if y is not None else None,
                                             _ptr(w_post) if w_post is not None else None, _ptr(w_pre),
                                             float(eps), _ptr(x_out) if x_out is not None else None, os_, ls,
                                             _stream())
    assert_cuda_ok(code, "matMulRmsNorm")
    return outs, x_out


def mat_mul_quantized(type_name: str, weight_bytes, input_columns, input_size: int, row_count: int,
                      column_count: int) -> np.ndarray:
    """wasm-kernels.ts:416-466 -> hp_matmul_quantized_f32 (lib.rs:41): host
    buffers in and out, nothing stays resident."""
    tid = quantized_type_id(type_name)
    w = np.ascontiguousarray(np.frombuffer(weight_bytes, dtype=np.uint8)
                             if isinstance(weight_bytes, (bytes, bytearray, memoryview)) else weight_bytes,
                             dtype=np.uint8)
    x = np.ascontiguousarray(input_columns, dtype=np.float32)
    if x.size != input_size * column_count:
        raise CudaKernelError(ERR_SHAPE, f"Quantized matmul input shape mismatch: {x.size}")
    out = np.empty(row_count * column_count, np.float32)
    code = _lib.lib().hpc_matmul_quantized_f32(tid, w.ctypes.data_as(C.c_void_p), w.size,
                                               x.ctypes.data_as(C.c_void_p), x.size, input_size, row_count,
                                               column_count, out.ctypes.data_as(C.c_void_p), out.size)
    assert_cuda_ok(code, "matMulQuantized")
    return out


def mat_mul_dequantized(type_name: str, weight_bytes, input_columns, input_size: int, row_count: int,
                        column_count: int) -> np.ndarray:
    """wasm-kernels.ts:468-520 matMulDequantizedWasm -> hp_matmul_dequantized_f32
    (lib.rs:103-154): bit-exact dequantized rows times the input columns with
    the reference's sequential f32 sum; host buffers in and out."""
    tid = quantized_type_id(type_name)
    w = np.ascontiguousarray(np.frombuffer(weight_bytes, dtype=np.uint8)
                             if isinstance(weight_bytes, (bytes, bytearray, memoryview)) else weight_bytes,
                             dtype=np.uint8)
    x = np.ascontiguousarray(input_columns, dtype=np.float32)
    if x.size != input_size * column_count:
        raise CudaKernelError(ERR_SHAPE, f"Dequantized matmul input shape mismatch: {x.size}")
    out = np.empty(row_count * column_count, np.float32)
    code = _lib.lib().hpc_matmul_dequantized_f32(tid, w.ctypes.data_as(C.c_void_p), w.size,
                                                 x.ctypes.data_as(C.c_void_p), x.size, input_size, row_count,
                                                 column_count, out.ctypes.data_as(C.c_void_p), out.size)
    assert_cuda_ok(code, "matMulDequantized")
    return out


def mat_mul_dequantized_resident(handle: CudaQuantizedWeightHandle, input_columns, input_size: int, row_count: int,
                                 column_count: int):
    """The same arithmetic on a resident weight (hpc_matmul_dequantized_prepared_f32)."""
    x, from_host = _as_device_f32(input_columns)
    out = torch.empty(row_count * column_count, dtype=torch.float32, device="cuda")
    code = _lib.lib().hpc_matmul_dequantized_prepared_f32(handle.handle, _ptr(x), x.numel(), input_size, row_count,
                                                          column_count, _ptr(out), out.numel(), _stream())
    assert_cuda_ok(code, "matMulDequantizedResident")
    return out.cpu().numpy() if from_host else out


def lm_head_topk(handle: CudaQuantizedWeightHandle, hidden, column_count: int, k: int, *, softcap: float = 0.0,
                 id_offset: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Fused LM head + top-k on normed hidden columns: (ids, values), each
    [column_count, k], ordered by value descending then id ascending
    (runtime.ts:514-527).  softcap > 0 applies fround(tanh(v/c)*c) after
    selection (mergeTopCandidates, webgpu/segment-runner.ts:3773-3794)."""
    x, from_host = _as_device_f32(hidden)
    if x.numel() != handle.input_size * column_count:
        raise CudaKernelError(ERR_SHAPE, f"LM head hidden shape mismatch: {x.numel()}")
    ids = torch.empty((column_count, k), dtype=torch.int32, device="cuda")
    vals = torch.empty((column_count, k), dtype=torch.float32, device="cuda")
    code = _lib.lib().hpc_lm_head_topk(handle.handle, _ptr(x), x.numel(), handle.input_size, column_count, k,
                                       id_offset, softcap, _ptr(ids), _ptr(vals), _stream())
    assert_cuda_ok(code, "lmHeadTopK")
    if from_host:
        return ids.cpu(), vals.cpu()
    return ids, vals


def sample_candidates(ids: torch.Tensor, vals: torch.Tensor, *, top_k: int, top_p: float, temperature: float,
                      greedy: bool, rng_state: int, token_out: torch.Tensor, table: torch.Tensor | None = None,
                      scale: float = 1.0, row_out: torch.Tensor | None = None) -> None:
    """The sampler's token draw on the device (hpc_sample_candidates): ids /
    vals a sorted candidate list (device int32 / f32), token_out a device
    int32 slot; with `table` ([rows][hidden] f32) the chosen row * scale goes
    to row_out.  Nothing is read back (no synchronization)."""
    if ids.dtype != torch.int32 or vals.dtype != torch.float32 or not ids.is_cuda or not vals.is_cuda:
        raise CudaKernelError(ERR_TYPE, "sample: candidates must be device int32 ids and f32 values")
    n = ids.numel()
    rows, hidden = (table.shape[0], table.shape[1]) if table is not None else (0, 0)
    if table is not None and (row_out is None or row_out.numel() < hidden or table.dtype != torch.float32
                              or not table.is_contiguous()):
        raise CudaKernelError(ERR_SHAPE, "sample: the table must be contiguous f32 and row_out hold a row")
    code = _lib.lib().hpc_sample_candidates(_ptr(ids), _ptr(vals), n, max(1, int(top_k)), float(top_p),
                                            float(temperature), 1 if greedy else 0, int(rng_state) & 0xFFFFFFFF,
                                            _ptr(token_out), _ptr(table) if table is not None else None, rows,
                                            hidden, float(scale), _ptr(row_out) if row_out is not None else None,
                                            _stream())
    assert_cuda_ok(code, "sampleCandidates")


def set_matmul_order(exact: bool) -> None:
    """Reference f32 order (default) or the reordered kernels for the matmul
    and LM-head calls (hpc_set_matmul_order)."""
    assert_cuda_ok(_lib.lib().hpc_set_matmul_order(int(bool(exact))), "setMatmulOrder")


def device_error() -> None:
    """Raises CudaKernelError(ERR_TIMEOUT) if a kernel's bounded wait gave up."""
    assert_cuda_ok(_lib.lib().hpc_device_error(), "deviceStatus")
