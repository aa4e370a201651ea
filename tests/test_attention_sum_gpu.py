"""The exact attention's softmax sum (hc_attx.cu seq_sum_nonneg_warp).

lib.rs:627-635 adds the probabilities one by one in f32.  The GPU computes
that same sequential sum with a warp: exact integer prefix scans while the
running sum stays in one binade, one real f32 add at every binade change or
exact tie.  Here it must equal a plain sequential float32 sum
(numpy add.accumulate) bit for bit on inputs chosen to exercise every branch:
softmax-like terms, long runs of half-ulp ties (round half to even), binade
crossings at every step, subnormals and zeros, and every length around the
warp's 256-term blocks.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def hook():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from heliopause_b200 import _lib
    from heliopause_b200 import kernels as hk
    hk.init_device(0)
    f = _lib.lib().hc_test_seq_sum
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    return f


def _run(hook, v):
    v = np.ascontiguousarray(v, np.float32)
    d = torch.from_numpy(v).cuda()
    out = torch.zeros(1, device="cuda")
    assert hook(C.c_void_p(d.data_ptr()), v.size, C.c_void_p(out.data_ptr())) == 0
    got = out.cpu().numpy()[0]
    ref = np.add.accumulate(v, dtype=np.float32)[-1] if v.size else np.float32(0.0)
    assert got.view(np.uint32) == np.float32(ref).view(np.uint32), f"{got!r} vs {ref!r}"


def _cases():
    g = np.random.default_rng(11)
    s = g.normal(0, 16, 4096).astype(np.float32)
    yield "softmax", np.exp((s - s.max()).astype(np.float64)).astype(np.float32)
    yield "softmax-flat", np.exp(g.normal(0, 1, 4096) - 4).astype(np.float32)
    yield "uniform", g.random(4096, dtype=np.float32)
    yield "ones", np.ones(4096, np.float32)  # a binade change at every power of two
    yield "half-ulp ties", np.concatenate([[1.0], np.full(3000, 2.0 ** -24)]).astype(np.float32)
    yield "odd ties", np.concatenate([[1.0 + 2.0 ** -23], np.full(3000, 2.0 ** -24)]).astype(np.float32)
    yield "mixed ties", np.tile(np.array([1.0, 2.0 ** -24, 3 * 2.0 ** -25, 2.0 ** -23], np.float32), 1024)
    yield "subnormal", np.concatenate([np.full(500, 1e-45), np.full(500, 3e-39), [1e-30],
                                       np.full(500, 1e-45)]).astype(np.float32)
    yield "zeros", np.zeros(300, np.float32)
    yield "zeros then one", np.concatenate([np.zeros(700), [1.0], np.zeros(10)]).astype(np.float32)
    yield "rising", (np.arange(4096, dtype=np.float32) / 4096.0) ** 8
    yield "spikes", np.where(g.random(4096) < 0.01, 1.0, g.random(4096) * 1e-6).astype(np.float32)


@pytest.mark.parametrize("name", [c[0] for c in _cases()])
def test_warp_sum_equals_sequential_sum(hook, name):
    _run(hook, dict(_cases())[name])


@pytest.mark.parametrize("n", [1, 2, 31, 255, 256, 257, 511, 4095, 4096])
def test_every_length(hook, n):
    g = np.random.default_rng(n)
    _run(hook, np.exp(g.normal(0, 3, n) - 6).astype(np.float32))
