"""ctypes wrapper around the C restatement of the Heliopause hot path.

TEST INFRASTRUCTURE ONLY: the parity oracle and the timed CPU baseline.  Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py`` import
this module.  The CUDA product path never does.

Parity pinning: the restated functions are checked against every known-answer
vector the reference's own tests hold for this path (f16 codec, Q8_0/Q4_0
block dequant, block byte sizes, the Q4_0 matmul fixture, the RNG first draw,
the synthetic forward top-2) and against gguf-py 0.19.0's independent numpy
dequantizers for Q4_K/Q6_K (tests/test_oracle_pins.py).  No reference test
pins Q4_K/Q6_K dot products, so those rest on the line-by-line restatement of
packages/engine/wasm-kernels/src/lib.rs:1877-2172.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "libhp_oracle.so"

Q4_K, Q5_K, Q6_K, IQ4_XS, Q8_0, Q4_0 = 1, 2, 3, 4, 5, 6
TYPE_IDS = {"Q4_K": Q4_K, "Q5_K": Q5_K, "Q6_K": Q6_K, "IQ4_XS": IQ4_XS, "Q8_0": Q8_0, "Q4_0": Q4_0}
BLOCK_BYTES = {Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210), IQ4_XS: (256, 136), Q8_0: (32, 34), Q4_0: (32, 18)}

OK, ERR_SHAPE, ERR_HEADS, ERR_TYPE = 0, 1, 2, 3

_f32p = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_i8p = C.POINTER(C.c_int8)
_i16p = C.POINTER(C.c_int16)
_i32p = C.POINTER(C.c_int32)
_sz = C.c_size_t


def build() -> Path:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        L = C.CDLL(str(_LIB_PATH))
        L.hpo_f16_to_f32.restype = C.c_float
        L.hpo_f16_to_f32.argtypes = [C.c_uint16]
        L.hpo_f32_to_f16_rust.restype = C.c_uint16
        L.hpo_f32_to_f16_rust.argtypes = [C.c_float]
        L.hpo_f32_to_f16_ts.restype = C.c_uint16
        L.hpo_f32_to_f16_ts.argtypes = [C.c_float]
        L.hpo_dequantize_row.restype = C.c_int
        L.hpo_dequantize_row.argtypes = [C.c_int, _u8p, _sz, _sz, _f32p]
        L.hpo_quantize_q8_k.argtypes = [_f32p, _sz, _f32p, _i8p, _i16p]
        L.hpo_quantize_q8_0.argtypes = [_f32p, _sz, _f32p, _i8p]
        L.hpo_matmul_quantized_f32.argtypes = [C.c_int, _u8p, _sz, _f32p, _sz, _sz, _sz, _sz, _f32p, _sz]
        L.hpo_matmul_dequantized_f32.argtypes = [C.c_int, _u8p, _sz, _f32p, _sz, _sz, _sz, _sz, _f32p, _sz]
        L.hpo_prepare_quantized_scales_f32.argtypes = [C.c_int, _u8p, _sz, _sz, _sz, _f32p, _sz]
        L.hpo_matmul_quantized_prepared_f32.argtypes = [C.c_int, _u8p, _sz, _f32p, _sz, _f32p, _sz, _sz, _sz, _sz, _f32p, _sz]
        L.hpo_matmul_prepared_threaded.argtypes = [C.c_int, _u8p, _sz, _f32p, _sz, _f32p, _sz, _sz, _sz, _sz, _f32p, _sz, C.c_int]
        L.hpo_matmul_multi_f32.argtypes = [_sz, _f32p, _sz, _sz, _sz, C.c_void_p, C.c_int]
        L.hpo_split_rows.restype = _sz
        L.hpo_split_rows.argtypes = [_sz, _sz, C.POINTER(_sz), C.POINTER(_sz)]
        L.hpo_gqa_attention_f32.argtypes = [_f32p, _sz, _f32p, _sz, _f32p, _sz, _f32p, _sz, _sz, _sz, _sz, _sz, _sz,
                                            _sz, _sz, C.c_float, C.c_int, C.c_int, _f32p, _sz]
        L.hpo_topk.restype = _sz
        L.hpo_topk.argtypes = [_f32p, _sz, _sz, _i32p, _f32p]
        L.hpo_rms_norm_rows.argtypes = [_f32p, _sz, _sz, _f32p, C.c_double, _f32p]
        L.hpo_rms_norm_rows_noweight.argtypes = [_f32p, _sz, _sz, C.c_double, _f32p]
        L.hpo_rope_neox.argtypes = [_f32p, _sz, _sz, _sz, _i32p, _sz, C.c_double, _f32p, _f32p]
        L.hpo_cast_f16_rows.argtypes = [_f32p, _sz, _f32p]
        L.hpo_gelu.restype = C.c_double
        L.hpo_gelu.argtypes = [C.c_float]
        L.hpo_geglu.argtypes = [_f32p, _f32p, _sz, _f32p]
        L.hpo_softcap.argtypes = [_f32p, _sz, C.c_double]
        L.hpo_kv_update.argtypes = [_f32p, _f32p, _sz, _sz, _sz, _sz, _f32p, _f32p, _i32p, _sz]
        L.hpo_scale_embedding.argtypes = [_f32p, _sz, C.c_double]
        L.hpo_rms_norm_f32sum_rows.argtypes = [_f32p, _sz, _sz, _f32p, C.c_double, _f32p]
        L.hpo_rope_neox_pairs.argtypes = [_f32p, _sz, _sz, C.c_int32, _sz, _sz, C.c_double, _f32p]
        L.hpo_gelu_mul_f32.argtypes = [_f32p, _f32p, _sz, _f32p]
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(bytes(a), dtype=np.uint8) if isinstance(a, (bytes, bytearray)) else a,
                                dtype=np.uint8)


class OracleError(RuntimeError):
    def __init__(self, code: int, what: str):
        names = {1: "shape mismatch", 2: "head count mismatch", 3: "unsupported type"}
        super().__init__(f"{what} oracle {names.get(code, f'failed with code {code}')}")
        self.code = code


def _check(code: int, what: str) -> None:
    if code != OK:
        raise OracleError(code, what)


# ---------------------------------------------------------------- codecs ---

def f16_to_f32(h: int) -> float:
    return lib().hpo_f16_to_f32(h)


def f32_to_f16_rust(x: float) -> int:
    return lib().hpo_f32_to_f16_rust(x)


def f32_to_f16_ts(x: float) -> int:
    return lib().hpo_f32_to_f16_ts(x)


def row_bytes(type_id: int, k: int) -> int:
    blk, nbytes = BLOCK_BYTES[type_id]
    return k // blk * nbytes


def dequantize(type_id: int, data, k: int, rows: int = 1) -> np.ndarray:
    data = _u8(data)
    rb = row_bytes(type_id, k)
    out = np.empty((rows, k), np.float32)
    for r in range(rows):
        seg = np.ascontiguousarray(data[r * rb:(r + 1) * rb])
        if not lib().hpo_dequantize_row(type_id, _p(seg, _u8p), rb, k, _p(out[r], _f32p)):
            raise OracleError(ERR_TYPE, "dequantize")
    return out


def quantize_q8_k(x) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    x = _f32(x)
    n = x.size
    d = np.empty(n // 256, np.float32)
    qs = np.empty(n, np.int8)
    bs = np.empty(n // 32, np.int16)
    lib().hpo_quantize_q8_k(_p(x, _f32p), n, _p(d, _f32p), _p(qs, _i8p), _p(bs, _i16p))
    return d, qs, bs


def quantize_q8_0(x) -> tuple[np.ndarray, np.ndarray]:
    x = _f32(x)
    n = x.size
    d = np.empty(n // 32, np.float32)
    qs = np.empty(n, np.int8)
    lib().hpo_quantize_q8_0(_p(x, _f32p), n, _p(d, _f32p), _p(qs, _i8p))
    return d, qs


# --------------------------------------------------------------- drivers ---

def matmul_quantized(type_id: int, weight, x, k: int, rows: int, cols: int) -> np.ndarray:
    """lib.rs:41-100 hp_matmul_quantized_f32; output [cols][rows]."""
    w = _u8(weight)
    x = _f32(x)
    out = np.empty(rows * cols, np.float32)
    _check(lib().hpo_matmul_quantized_f32(type_id, _p(w, _u8p), w.size, _p(x, _f32p), x.size, k, rows, cols,
                                          _p(out, _f32p), out.size), "matMulQuantized")
    return out


def prepare_scales(type_id: int, weight, k: int, rows: int) -> np.ndarray:
    w = _u8(weight)
    per_row = {Q4_K: 2, Q5_K: 2}.get(type_id, 1) * (k // BLOCK_BYTES[type_id][0])
    s = np.empty(per_row * rows, np.float32)
    _check(lib().hpo_prepare_quantized_scales_f32(type_id, _p(w, _u8p), w.size, k, rows, _p(s, _f32p), s.size),
           "prepareQuantizedScales")
    return s


def matmul_prepared(type_id: int, weight, scales, x, k: int, rows: int, cols: int, threads: int = 1) -> np.ndarray:
    """lib.rs:225-298 hp_matmul_quantized_prepared_f32 (threads > 1 row-shards
    the rows like the WASM thread pool; the results are identical)."""
    w = _u8(weight)
    s = _f32(scales)
    x = _f32(x)
    out = np.empty(rows * cols, np.float32)
    if threads <= 1:
        code = lib().hpo_matmul_quantized_prepared_f32(type_id, _p(w, _u8p), w.size, _p(s, _f32p), s.size,
                                                       _p(x, _f32p), x.size, k, rows, cols, _p(out, _f32p), out.size)
    else:
        code = lib().hpo_matmul_prepared_threaded(type_id, _p(w, _u8p), w.size, _p(s, _f32p), s.size,
                                                  _p(x, _f32p), x.size, k, rows, cols, _p(out, _f32p), out.size,
                                                  threads)
    _check(code, "matMulQuantizedResident")
    return out


class _Spec(C.Structure):
    _fields_ = [("type", C.c_int), ("w", C.c_void_p), ("wlen", C.c_size_t), ("scales", C.c_void_p),
                ("slen", C.c_size_t), ("rows", C.c_size_t), ("out", C.c_void_p), ("outlen", C.c_size_t)]


def matmul_multi(specs, x, k: int, cols: int, prepared: bool = True) -> list[np.ndarray]:
    """lib.rs:302-426 / 430-536.  specs: list of (type_id, weight, scales|None, rows)."""
    x = _f32(x)
    keep = []
    arr = (_Spec * max(1, len(specs)))()
    outs = []
    for i, (t, w, s, rows) in enumerate(specs):
        w = _u8(w)
        s = _f32(s) if s is not None else np.zeros(1, np.float32)
        o = np.empty(rows * cols, np.float32)
        keep += [w, s]
        outs.append(o)
        arr[i] = _Spec(t, w.ctypes.data, w.size, s.ctypes.data, s.size if prepared else 0, rows, o.ctypes.data, o.size)
    _check(lib().hpo_matmul_multi_f32(len(specs), _p(x, _f32p), x.size, k, cols, C.cast(arr, C.c_void_p),
                                      1 if prepared else 0), "matMulQuantizedMulti")
    return outs


def matmul_dequantized(type_id: int, weight, x, k: int, rows: int, cols: int) -> np.ndarray:
    w = _u8(weight)
    x = _f32(x)
    out = np.empty(rows * cols, np.float32)
    _check(lib().hpo_matmul_dequantized_f32(type_id, _p(w, _u8p), w.size, _p(x, _f32p), x.size, k, rows, cols,
                                            _p(out, _f32p), out.size), "matMulDequantized")
    return out


def split_rows(rows: int, shards: int) -> list[tuple[int, int]]:
    st = (_sz * shards)()
    ct = (_sz * shards)()
    n = lib().hpo_split_rows(rows, shards, st, ct)
    return [(st[i], ct[i]) for i in range(n)]


def gqa_attention(q, key, value, *, head, nq, nkv, ntok, nkvtok, kvstart, cap, scale, value_layout, qf16,
                  mask=None) -> np.ndarray:
    q = _f32(q)
    key = _f32(key)
    value = _f32(value)
    m = _f32(mask) if mask is not None else np.zeros(0, np.float32)
    out = np.empty(ntok * nq * head, np.float32)
    _check(lib().hpo_gqa_attention_f32(_p(q, _f32p), q.size, _p(key, _f32p), key.size, _p(value, _f32p), value.size,
                                       _p(m, _f32p), m.size, head, nq, nkv, ntok, nkvtok, kvstart, cap, scale,
                                       value_layout, 1 if qf16 else 0, _p(out, _f32p), out.size), "gqaAttention")
    return out


def topk(values, k: int) -> tuple[np.ndarray, np.ndarray]:
    """runtime.ts:514-527 (value descending, lower id first on ties)."""
    v = _f32(values)
    ids = np.empty(k, np.int32)
    vals = np.empty(k, np.float32)
    n = lib().hpo_topk(_p(v, _f32p), v.size, k, _p(ids, _i32p), _p(vals, _f32p))
    return ids[:n].copy(), vals[:n].copy()


# ----------------------------------------------------------- decoder math ---

def rms_norm_rows(x, w, eps: float) -> np.ndarray:
    x = _f32(x)
    w = _f32(w)
    o = np.empty_like(x)
    lib().hpo_rms_norm_rows(_p(x, _f32p), x.size // w.size, w.size, _p(w, _f32p), eps, _p(o, _f32p))
    return o


def rms_norm_rows_noweight(x, dim: int, eps: float) -> np.ndarray:
    x = _f32(x)
    o = np.empty_like(x)
    lib().hpo_rms_norm_rows_noweight(_p(x, _f32p), x.size // dim, dim, eps, _p(o, _f32p))
    return o


def rope_neox(x, head: int, nheads: int, positions, ndims: int, freq_base: float, factors=None) -> np.ndarray:
    x = _f32(x)
    pos = np.ascontiguousarray(positions, np.int32)
    o = np.empty_like(x)
    f = _f32(factors) if factors is not None else None
    lib().hpo_rope_neox(_p(x, _f32p), head, nheads, pos.size, _p(pos, _i32p), ndims, freq_base,
                        _p(f, _f32p) if f is not None else None, _p(o, _f32p))
    return o


def cast_f16_rows(x) -> np.ndarray:
    x = _f32(x)
    o = np.empty_like(x)
    lib().hpo_cast_f16_rows(_p(x, _f32p), x.size, _p(o, _f32p))
    return o


def geglu(gate, up) -> np.ndarray:
    g = _f32(gate)
    u = _f32(up)
    o = np.empty_like(g)
    lib().hpo_geglu(_p(g, _f32p), _p(u, _f32p), g.size, _p(o, _f32p))
    return o


def softcap(x, cap: float) -> np.ndarray:
    o = _f32(x).copy()
    lib().hpo_softcap(_p(o, _f32p), o.size, cap)
    return o


def kv_update(kc: np.ndarray, vc: np.ndarray, cap: int, nkv: int, klen: int, vlen: int, k, v, positions) -> None:
    k = _f32(k)
    v = _f32(v)
    pos = np.ascontiguousarray(positions, np.int32)
    assert kc.dtype == np.float32 and vc.dtype == np.float32 and kc.flags.c_contiguous and vc.flags.c_contiguous
    lib().hpo_kv_update(_p(kc, _f32p), _p(vc, _f32p), cap, nkv, klen, vlen, _p(k, _f32p), _p(v, _f32p),
                        _p(pos, _i32p), pos.size)


def scale_embedding(x, dim: int) -> np.ndarray:
    o = _f32(x).copy()
    lib().hpo_scale_embedding(_p(o, _f32p), o.size, float(dim))
    return o


# ------------------------------------------------------ MTP draft head math ---

def rms_norm_f32sum_rows(x, w, eps: float) -> np.ndarray:
    """mtp-assistant-runner.ts:275-290 rmsNorm (f32 sum of squares)."""
    x = _f32(x)
    w = _f32(w)
    o = np.empty_like(x)
    lib().hpo_rms_norm_f32sum_rows(_p(x, _f32p), x.size // w.size, w.size, _p(w, _f32p), eps, _p(o, _f32p))
    return o


def rope_neox_pairs(x, head: int, nheads: int, position: int, ndims: int, pairs: int, freq_base: float) -> np.ndarray:
    """mtp-assistant-runner.ts:361-387 ropeNeox with activePairCount."""
    x = _f32(x)
    o = np.empty_like(x)
    lib().hpo_rope_neox_pairs(_p(x, _f32p), head, nheads, position, ndims, pairs, freq_base, _p(o, _f32p))
    return o


def gelu_mul_f32(gate, up) -> np.ndarray:
    """mtp-assistant-runner.ts:150-153 + 399-411: fround(gelu(gate) * up)."""
    g = _f32(gate)
    u = _f32(up)
    o = np.empty_like(g)
    lib().hpo_gelu_mul_f32(_p(g, _f32p), _p(u, _f32p), g.size, _p(o, _f32p))
    return o


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0))
