"""The C-ABI library loads and exports every symbol the public header
declares; argument validation answers with the reference's status codes
before any device work (lib.rs:7-10).  Runs on CPU."""
import ctypes as C

import numpy as np
import pytest

from heliopause_b200 import _lib, kernels


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    declared = _lib.header_symbols()
    assert declared, "no hpc_* declarations found in include/*.h"
    missing = [n for n in declared if not hasattr(L, n)]
    assert not missing, f"declared but not exported: {missing}"
    # and the ctypes table covers the same set
    assert sorted(_lib.SIGNATURES) == declared


def test_version():
    assert _lib.lib().hpc_version() >> 16 == 1


def test_shape_errors_precede_device_work():
    L = _lib.lib()
    # input length != input_size * column_count -> ERR_SHAPE, whatever the handle
    assert L.hpc_matmul_quantized_prepared_f32(None, None, 5, 256, 4, 1, None, 4, None) == kernels.ERR_SHAPE
    assert L.hpc_matmul_quantized_prepared_multi_f32(0, None, 0, 256, 0, None, None, None, None) == kernels.ERR_SHAPE
    assert L.hpc_matmul_quantized_prepared_multi_f32(9, None, 0, 256, 0, None, None, None, None) == kernels.ERR_SHAPE
    w = np.zeros(144, np.uint8)
    x = np.zeros(256, np.float32)
    o = np.zeros(1, np.float32)
    vp = lambda a: a.ctypes.data_as(C.c_void_p)
    # unsupported type id -> ERR_TYPE (lib.rs:58-61)
    assert L.hpc_matmul_quantized_f32(42, vp(w), 144, vp(x), 256, 256, 1, 1, vp(o), 1) == kernels.ERR_TYPE
    # weight length mismatch -> ERR_SHAPE (lib.rs:62-64)
    assert L.hpc_matmul_quantized_f32(1, vp(w), 143, vp(x), 256, 256, 1, 1, vp(o), 1) == kernels.ERR_SHAPE
    # input size not a multiple of 256 for a K-quant -> ERR_TYPE (row_bytes is None)
    assert L.hpc_matmul_quantized_f32(1, vp(w), 144, vp(x), 200, 200, 1, 1, vp(o), 1) == kernels.ERR_TYPE
    # the dequantized matmul answers in the order of hp_matmul_dequantized_f32 (lib.rs:115-125)
    assert L.hpc_matmul_dequantized_f32(1, vp(w), 144, vp(x), 255, 256, 1, 1, vp(o), 1) == kernels.ERR_SHAPE
    assert L.hpc_matmul_dequantized_f32(42, vp(w), 144, vp(x), 256, 256, 1, 1, vp(o), 1) == kernels.ERR_TYPE
    assert L.hpc_matmul_dequantized_f32(3, vp(w), 144, vp(x), 256, 256, 1, 1, vp(o), 1) == kernels.ERR_SHAPE
    assert L.hpc_matmul_dequantized_prepared_f32(None, None, 5, 256, 4, 1, None, 4, None) == kernels.ERR_SHAPE
    assert L.hpc_matmul_dequantized_prepared_f32(None, None, 256, 256, 4, 1, None, 4, None) == kernels.ERR_ARG
    h = C.c_void_p()
    assert L.hpc_weight_upload(5, vp(w), 34, 32, 1, C.byref(h)) == kernels.ERR_TYPE  # Q8_0 is not resident
    assert L.hpc_weight_upload(1, vp(w), 100, 256, 1, C.byref(h)) == kernels.ERR_SHAPE
    assert L.hpc_weight_release(None) == kernels.ERR_ARG
    assert "invalid weight handle" in _lib.last_error()


def test_assert_cuda_ok_messages():
    with pytest.raises(kernels.CudaKernelError, match="x cuda shape mismatch"):
        kernels.assert_cuda_ok(kernels.ERR_SHAPE, "x")
    with pytest.raises(kernels.CudaKernelError, match="x cuda unsupported type"):
        kernels.assert_cuda_ok(kernels.ERR_TYPE, "x")
    with pytest.raises(kernels.CudaKernelError, match="code 4"):
        kernels.assert_cuda_ok(kernels.ERR_CUDA, "x")
    kernels.assert_cuda_ok(kernels.OK, "x")
    assert kernels.quantized_type_id("Q4_K") == 1 and kernels.quantized_type_id("Q6_K") == 3


# ---- prototypes in include/*.h against the ctypes table -----------------------

_C_SCALARS = {"size_t": ("u", 8), "int": ("i", 4), "int32_t": ("i", 4), "uint32_t": ("u", 4),
              "int64_t": ("i", 8), "uint64_t": ("u", 8), "float": ("f", 4), "double": ("f", 8)}
_C_HANDLES = {"hpc_weight", "hpc_model", "hpc_draft"}  # typedefs of struct pointers


def _header_prototypes():
    """name -> (return type, [parameter declarations]) for every hpc_* prototype."""
    import re
    protos = {}
    for h in _lib.HEADERS:
        src = h.read_text()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        src = re.sub(r"^[ \t]*#[^\n]*", "", src, flags=re.M)
        for ret, name, params in re.findall(r"([A-Za-z_][\w\s*]*?)\b(hpc_\w+)\s*\(([^)]*)\)\s*;", src):
            ps = [" ".join(p.split()) for p in params.split(",")]
            protos[name] = (" ".join(ret.split()), [] if ps in (["void"], [""]) else ps)
    return protos


def _c_kind(decl):
    """'p' for pointers and handles, else (signedness/float, bytes)."""
    if "*" in decl:
        return "p"
    words = [w for w in decl.split() if w not in ("const", "volatile")]
    base = words[0] if len(words) == 1 else " ".join(words[:-1])  # drop the parameter name
    if base in _C_HANDLES:
        return "p"
    assert base in _C_SCALARS, f"unclassified C type {base!r} in {decl!r}"
    return _C_SCALARS[base]


def _ctypes_kind(t):
    if t in (C.c_void_p, C.c_char_p) or (isinstance(t, type) and issubclass(t, C._Pointer)):
        return "p"
    if t in (C.c_float, C.c_double):
        return ("f", C.sizeof(t))
    return ("i" if t(-1).value < 0 else "u", C.sizeof(t))


def test_ctypes_signatures_match_header_prototypes():
    protos = _header_prototypes()
    assert sorted(protos) == _lib.header_symbols()
    bad = []
    for name, (res, args) in _lib.SIGNATURES.items():
        ret, params = protos[name]
        if len(params) != len(args):
            bad.append(f"{name}: {len(params)} parameters in the header, {len(args)} in ctypes")
            continue
        if _c_kind(ret + " r") != _ctypes_kind(res):
            bad.append(f"{name}: return {ret!r} vs {res}")
        for i, (decl, t) in enumerate(zip(params, args)):
            if _c_kind(decl) != _ctypes_kind(t):
                bad.append(f"{name} arg {i} {decl!r}: {_c_kind(decl)} vs ctypes {t} {_ctypes_kind(t)}")
    assert not bad, "\n".join(bad)


def test_model_create_rejects_attention_wider_than_shared_memory():
    # An attention CTA stages the queries of every token of a step for its KV
    # head (1,280 bytes each beside 130 KB of K/V rows), so 16 query heads per
    # KV head at 8 tokens per step cannot fit the kernels' 220 KB: rejected at
    # create time, before any device work, instead of failing in a forward.
    cfg = _lib.ModelConfig(hidden=4096, heads=16, kv_heads=1, head_dim=256, ffn=2048, vocab=4096, layers=1,
                           kv_layers=1, context=64, max_tokens=8, top_k=8, rms_eps=1e-6, rope_theta=1e4,
                           final_logit_softcap=0.0)
    out = C.c_void_p()
    assert _lib.lib().hpc_model_create(C.byref(cfg), C.byref(out)) == kernels.ERR_SHAPE
    assert "attention shared memory" in _lib.last_error()
    assert not out.value
