"""hpc_lm_head_topk_noalloc (static device scratch, no allocation in the
call) against hpc_lm_head_topk (cudaMallocAsync scratch), both through the
C-ABI.  Two calls in a row on different inputs each match the allocating
entry point (ids exactly, values within rtol 1e-3 / atol 1e-4), so what a
call leaves in the shared scratch does not leak into the next one.  A call
whose scratch exceeds HPC_NOALLOC_SCRATCH_BYTES is refused with
HPC_ERR_SHAPE before any launch, and the widest call that still fits
matches the allocating entry point.  Collected last (file name) and
independent of the other test files' state.
"""
import ctypes as C

import numpy as np
import pytest

from heliopause_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 4 << 20  # HPC_NOALLOC_SCRATCH_BYTES


@pytest.fixture(scope="module")
def env():
    import torch

    from heliopause_b200 import _lib
    from heliopause_b200 import kernels as hk
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    hk.init_device(0)
    return torch, hk, _lib.lib()


def _call(L, fn, torch, head, x, cols, k, softcap):
    ids = torch.full((cols * k,), -1, dtype=torch.int32, device="cuda")
    vals = torch.full((cols * k,), float("nan"), device="cuda")
    rc = getattr(L, fn)(head.handle, C.c_void_p(x.data_ptr()), x.numel(), head.input_size, cols, k, 0,
                        C.c_float(softcap), C.c_void_p(ids.data_ptr()), C.c_void_p(vals.data_ptr()),
                        C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, L.hpc_last_error()
    torch.cuda.synchronize()
    return ids.cpu().numpy().reshape(cols, k), vals.cpu().numpy().reshape(cols, k)


def test_noalloc_matches_allocating_entry_point_twice_in_a_row(env):
    torch, hk, L = env
    kdim, rows, k = 2048, 262144, 40
    head = hk.create_quantized_weight_handle("Q6_K", syn.q6_k_weight(rows, kdim, seed=4242), kdim, rows)
    try:
        for cols, seed, softcap in ((5, 11, 0.0), (1, 12, 30.0)):
            x = torch.from_numpy(syn.activations(cols, kdim, seed=seed)).cuda()
            ids, vals = _call(L, "hpc_lm_head_topk_noalloc", torch, head, x, cols, k, softcap)
            rids, rvals = _call(L, "hpc_lm_head_topk", torch, head, x, cols, k, softcap)
            assert np.array_equal(ids, rids)
            assert np.all(np.abs(vals.astype(np.float64) - rvals) <= 1e-4 + 1e-3 * np.abs(rvals))
    finally:
        hk.release_quantized_weight_handle(head)


def test_noalloc_at_its_size_limit(env):
    # The widest call that still fits the static scratch (Q8_K records plus
    # candidate lists within HPC_NOALLOC_SCRATCH_BYTES), found by the entry
    # point's own answers, matches the allocating entry point -- so the carve
    # at the array's upper end is right -- and one column more is refused
    # with HPC_ERR_SHAPE before any launch.
    torch, hk, L = env
    kdim, rows, k = 256, 65536, 64
    head = hk.create_quantized_weight_handle("Q6_K", syn.q6_k_weight(rows, kdim, seed=7), kdim, rows)
    try:
        def rc(cols):
            x = torch.zeros(cols * kdim, device="cuda")
            ids = torch.empty(cols * k, dtype=torch.int32, device="cuda")
            vals = torch.empty(cols * k, device="cuda")
            r = L.hpc_lm_head_topk_noalloc(head.handle, C.c_void_p(x.data_ptr()), x.numel(), kdim, cols, k, 0,
                                           C.c_float(0.0), C.c_void_p(ids.data_ptr()), C.c_void_p(vals.data_ptr()),
                                           None)
            torch.cuda.synchronize()
            return r

        lo, hi = 1, 2
        while rc(hi) == 0:  # grow until refused
            lo, hi = hi, hi * 2
        while hi - lo > 1:  # largest fitting width in (lo, hi)
            mid = (lo + hi) // 2
            if rc(mid) == 0:
                lo = mid
            else:
                hi = mid
        fit = lo
        assert rc(fit + 1) == hk.ERR_SHAPE
        assert b"static" in L.hpc_last_error()
        x = torch.from_numpy(syn.activations(fit, kdim, seed=fit)).cuda()
        ids, vals = _call(L, "hpc_lm_head_topk_noalloc", torch, head, x, fit, k, 0.0)
        rids, rvals = _call(L, "hpc_lm_head_topk", torch, head, x, fit, k, 0.0)
        assert np.array_equal(ids, rids)
        assert np.all(np.abs(vals.astype(np.float64) - rvals) <= 1e-4 + 1e-3 * np.abs(rvals))
    finally:
        hk.release_quantized_weight_handle(head)
