"""Loads libheliocuda.so (built in-tree) and declares its C ABI for ctypes.

There is no CPU fallback: if the library or a CUDA device is missing, the
calls raise.  The declarations mirror include/heliocuda.h one for one.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libheliocuda.so"
HEADERS = sorted((PKG.parent / "include").glob("*.h"))

_sz = C.c_size_t
_vp = C.c_void_p
_i = C.c_int

# name -> (restype, argtypes)
SIGNATURES = {
    "hpc_last_error": (C.c_char_p, []),
    "hpc_version": (_i, []),
    "hpc_device_init": (_i, [_i]),
    "hpc_device_error": (_i, []),
    "hpc_set_matmul_order": (_i, [_i]),
    "hpc_set_wide_matmul_kind": (_i, [_i]),
    "hpc_weight_upload": (_i, [_i, _vp, _sz, _sz, _sz, C.POINTER(_vp)]),
    "hpc_weight_upload_device": (_i, [_i, _vp, _sz, _sz, _sz, _vp, C.POINTER(_vp)]),
    "hpc_weight_release": (_i, [_vp]),
    "hpc_weight_info": (_i, [_vp, C.POINTER(_i), C.POINTER(_sz), C.POINTER(_sz), C.POINTER(_sz)]),
    "hpc_weight_dequantize": (_i, [_vp, _vp, _sz, _vp]),
    "hpc_quantize_q8_k": (_i, [_vp, _sz, _sz, _sz, _vp, _vp, _vp, _vp]),
    "hpc_matmul_quantized_prepared_f32": (_i, [_vp, _vp, _sz, _sz, _sz, _sz, _vp, _sz, _vp]),
    "hpc_matmul_quantized_prepared_multi_f32": (_i, [_sz, _vp, _sz, _sz, _sz, C.POINTER(_vp), C.POINTER(_vp),
                                                     C.POINTER(_sz), _vp]),
    "hpc_matmul_quantized_f32": (_i, [_i, _vp, _sz, _vp, _sz, _sz, _sz, _sz, _vp, _sz]),
    "hpc_matmul_dequantized_f32": (_i, [_i, _vp, _sz, _vp, _sz, _sz, _sz, _sz, _vp, _sz]),
    "hpc_matmul_dequantized_prepared_f32": (_i, [_vp, _vp, _sz, _sz, _sz, _sz, _vp, _sz, _vp]),
    "hpc_q8_workspace_bytes": (_i, [_sz, _sz, C.POINTER(_sz)]),
    "hpc_q8_quantize": (_i, [_vp, _sz, _sz, _sz, _vp, _sz, _vp]),
    "hpc_matmul_q8": (_i, [_sz, C.POINTER(_vp), _vp, _sz, _sz, _sz, C.POINTER(_vp), C.POINTER(_sz), _vp]),
    "hpc_matmul_rmsnorm_f32": (_i, [_sz, C.POINTER(_vp), _vp, _sz, _sz, _sz, _vp, _vp, _vp, _vp, C.c_double, _vp,
                                    C.POINTER(_vp), C.POINTER(_sz), _vp]),
    "hpc_lm_head_topk": (_i, [_vp, _vp, _sz, _sz, _sz, _sz, C.c_int32, C.c_float, _vp, _vp, _vp]),
    "hpc_lm_head_topk_noalloc": (_i, [_vp, _vp, _sz, _sz, _sz, _sz, C.c_int32, C.c_float, _vp, _vp, _vp]),
    "hpc_lm_head_candidates_bytes": (_i, [_vp, _sz, _sz, C.POINTER(_sz)]),
    "hpc_lm_head_topk_q8": (_i, [_vp, _vp, _sz, _sz, _sz, _sz, C.c_int32, _vp, _sz, C.c_float, _vp, _vp, _vp, _vp]),
    "hpc_topk_merge_keys": (_i, [_vp, _sz, _sz, _sz, C.c_float, _vp, _vp, _vp]),
    "hpc_sample_candidates": (_i, [_vp, _vp, _sz, _sz, C.c_double, C.c_double, _i, C.c_uint32, _vp, _vp, _sz,
                                   _sz, C.c_double, _vp, _vp]),
    "hpc_model_create": (_i, [_vp, C.POINTER(_vp)]),
    "hpc_model_release": (_i, [_vp]),
    "hpc_model_set_weight": (_i, [_vp, _i, _i, _vp]),
    "hpc_model_set_norm": (_i, [_vp, _i, _i, _vp, _sz]),
    "hpc_model_set_lm_head": (_i, [_vp, _vp]),
    "hpc_model_set_exact": (_i, [_vp, _i]),
    "hpc_model_kv": (_i, [_vp, _i, C.POINTER(_vp), C.POINTER(_vp)]),
    "hpc_model_forward": (_i, [_vp, _vp, _vp, _sz, _sz, _vp, _vp, _vp, _vp]),
    "hpc_model_prefill": (_i, [_vp, _vp, _vp, _sz, _vp, _vp]),
    "hpc_draft_create": (_i, [_vp, C.POINTER(_vp)]),
    "hpc_draft_release": (_i, [_vp]),
    "hpc_draft_set_matrix": (_i, [_vp, _i, _i, _vp]),
    "hpc_draft_set_vector": (_i, [_vp, _i, _i, _vp, _sz]),
    "hpc_draft_set_layer_scale": (_i, [_vp, _i, C.c_float]),
    "hpc_draft_set_token_ordering": (_i, [_vp, _vp, _sz]),
    "hpc_draft_set_target_kv": (_i, [_vp, _i, _vp, _vp]),
    "hpc_draft_step": (_i, [_vp, _vp, _vp, _i, _sz, _vp, _vp, _vp, _vp]),
}


class ModelConfig(C.Structure):
    """hpc_model_config (include/heliocuda.h)."""
    _fields_ = [("hidden", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int), ("head_dim", C.c_int),
                ("ffn", C.c_int), ("vocab", C.c_int), ("layers", C.c_int), ("kv_layers", C.c_int),
                ("context", C.c_int), ("max_tokens", C.c_int), ("top_k", C.c_int), ("rms_eps", C.c_double),
                ("rope_theta", C.c_double), ("final_logit_softcap", C.c_float)]


class DraftConfig(C.Structure):
    """hpc_draft_config (include/heliocuda.h)."""
    _fields_ = [("backbone", C.c_int), ("hidden", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int), ("n_centroids", C.c_int),
                ("centroid_top_k", C.c_int), ("layers", C.c_int), ("context", C.c_int), ("max_top_k", C.c_int),
                ("rms_eps", C.c_double), ("rope_theta", C.c_double)]


_lib = None


class LibraryMissing(RuntimeError):
    pass


def header_symbols() -> list[str]:
    """Every function the public headers declare."""
    names = []
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"\b(hpc_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise LibraryMissing(f"{LIB_PATH} is not built; run `python -m heliopause_b200.build`")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().hpc_last_error().decode(errors="replace")
