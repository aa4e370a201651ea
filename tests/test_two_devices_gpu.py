"""One process driving two devices.

hpc_device_init selects the device per host thread, and kernel attributes
(the dynamic shared-memory limit, the carveout) belong to a device, so every
launcher sets them on each device at its first call there
(heliopause_b200/csrc/hc_once.h).  This runs matmuls whose launches need
more than the default 48 KB of dynamic shared memory -- the dp4a GEMV
(1 column), the tensor-core GEMV (5 columns) and the tensor-core matmul
(64 columns) -- on device 0 and then on device 1 from one process, and
checks every result against the C oracle within the north-star tolerance
(rtol 1e-3, atol 1e-4) and both devices' results against each other
(bit-identical: same kernels, same inputs).  Skips with fewer than two
devices.
"""
import numpy as np
import pytest
import torch

from heliopause_b200 import kernels as hk
from heliopause_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1e-4


@pytest.fixture(scope="module", autouse=True)
def _two_devices():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    yield
    hk.init_device(0)


def _matmul_on(dev, w, x, k, rows, cols):
    hk.init_device(dev)
    h = hk.create_quantized_weight_handle("Q4_K", w, k, rows)
    try:
        xd = torch.from_numpy(x).to(f"cuda:{dev}")
        out = hk.mat_mul_quantized_resident(h, xd, k, rows, cols)
        assert out.device.index == dev
        got = out.cpu().numpy()
    finally:
        hk.release_quantized_weight_handle(h)
    hk.device_error()
    return got


def _magnitude(oracle, w, x, k, rows, cols):
    """S = sum_i |w_i| * |x_q,i| per output, with the Q8_K-quantized input."""
    wd = np.abs(oracle.dequantize(syn.Q4_K, w, k, rows).astype(np.float64))
    out = []
    for c in range(cols):
        d, qs, _ = oracle.quantize_q8_k(x[c * k:(c + 1) * k])
        xa = np.abs(qs.astype(np.float64).reshape(-1, 256) * d.astype(np.float64)[:, None]).reshape(-1)
        out.append(wd @ xa)
    return np.concatenate(out)


@pytest.mark.parametrize("k,rows,cols", [(2048, 16384, 1), (2048, 16384, 5), (2048, 2048, 64)])
def test_same_process_two_devices(oracle, k, rows, cols):
    w = syn.quant_weight(syn.Q4_K, rows, k, seed=rows + cols)
    x = syn.activations(cols, k, seed=cols + 300)
    s = oracle.prepare_scales(syn.Q4_K, w, k, rows)
    ref = oracle.matmul_prepared(syn.Q4_K, w, s, x, k, rows, cols, threads=oracle.cpu_threads()).astype(np.float64)
    # the single-device tests' bound: north-star tolerance plus the f32
    # re-association term (nb + 8) * 2^-24 * S
    bound = ATOL + RTOL * np.abs(ref) + (k // 256 + 8) * 2.0 ** -24 * _magnitude(oracle, w, x, k, rows, cols)
    got0 = _matmul_on(0, w, x, k, rows, cols)
    got1 = _matmul_on(1, w, x, k, rows, cols)
    for dev, got in ((0, got0), (1, got1)):
        err = np.abs(got.astype(np.float64) - ref)
        assert np.all(err <= bound), f"device {dev}: max err {err.max():.3g}"
    assert np.array_equal(got0.view(np.uint32), got1.view(np.uint32))
