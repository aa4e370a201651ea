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
