"""GPU parity of the quantized matmul path against the C oracle.

  * dequantization of the resident (repacked) weights: bit-exact;
  * Q8_K activation quantization: bit-exact (d, qs, bsums);
  * matmul outputs in the default (reference) order, fewer than 16 columns:
    bit-exact -- every row dot keeps vec_dot_q*_k_q8_k_prepared's eight f32
    lane accumulators in block order (lib.rs:1924-1968, 2117-2172);
  * matmul outputs of the reordered kernels (hpc_set_matmul_order(0)) and of
    the tensor-core path (16+ columns): within the north-star tolerance
    rtol 1e-3 / atol 1e-4,
        |gpu - ref| <= 1e-4 + 1e-3 * |ref| + (nb + 8) * 2^-24 * S,
    on the configuration shapes (config 1: Q4_K 2048 -> 16384; config 2:
    Q/K/V/gate/up + Q6_K down, M in {1, 2, 4, 8}) and on ragged/edge shapes.
    The last term is the f32 re-association bound: both sides sum the same
    exact per-block integer products, the reference in 8 lane accumulators
    and the GPU in another fixed order, so for an output that is the small
    difference of large terms (S = sum_i |w_i * x_i|, nb = K/256 blocks) the
    two f32 results may legitimately differ by that much.  Every test reports
    how many outputs needed that term.
"""
import numpy as np
import pytest
import torch

from heliopause_b200 import kernels as hk
from heliopause_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-3, 1e-4


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    hk.init_device(0)


def _close(got, ref, mag=None, nb=8):
    """mag: S per output (sum |w*x| in f64); None -> strict north-star bound only."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    err = np.abs(got - ref)
    strict = ATOL + RTOL * np.abs(ref)
    bound = strict + (0.0 if mag is None else (nb + 8) * 2.0 ** -24 * mag)
    ok = err <= bound
    assert ok.all(), f"{(~ok).sum()} of {ok.size} outside tolerance; max err {err.max():.3g}"
    return int((err > strict).sum())


def _bitwise(got, ref, what):
    got = np.ascontiguousarray(got, np.float32)
    ref = np.ascontiguousarray(ref, np.float32)
    diff = got.view(np.uint32) != ref.view(np.uint32)
    assert not diff.any(), (f"{what}: {int(diff.sum())} of {diff.size} differ, max |d| "
                            f"{np.abs(got.astype(np.float64) - ref).max():.3g}")


def _magnitude(oracle, type_id, w, x, k, rows, cols):
    """S = sum_i |w_i| * |x_q,i| per output, with the Q8_K-quantized input."""
    wd = np.abs(oracle.dequantize(type_id, w, k, rows).astype(np.float64))
    out = []
    for c in range(cols):
        d, qs, _ = oracle.quantize_q8_k(x[c * k:(c + 1) * k])
        xa = np.abs(qs.astype(np.float64).reshape(-1, 256) * d.astype(np.float64)[:, None]).reshape(-1)
        out.append(wd @ xa)
    return np.concatenate(out)


TNAME = {syn.Q4_K: "Q4_K", syn.Q6_K: "Q6_K"}


@pytest.mark.parametrize("type_id", [syn.Q4_K, syn.Q6_K])
@pytest.mark.parametrize("rows,k", [(1, 256), (40, 512), (64, 2048), (33, 16384)])
def test_dequant_bit_exact(oracle, type_id, rows, k):
    w = syn.quant_weight(type_id, rows, k, seed=rows + k)
    h = hk.create_quantized_weight_handle(TNAME[type_id], w, k, rows)
    try:
        got = hk.dequantize_resident(h).cpu().numpy()
    finally:
        hk.release_quantized_weight_handle(h)
    ref = oracle.dequantize(type_id, w, k, rows)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_q8_k_quantize_bit_exact(oracle):
    k, cols = 2048, 5
    x = syn.activations(cols, k, seed=77)
    x[0:256] = 0.0                       # all-zero block
    x[256:512] = 1.0                     # all equal: first index wins
    x[512 + 10], x[512 + 200] = -4.0, 4.0  # tie across lanes, negative first
    x[768:1024] *= 1e-30                 # tiny values
    x[1024:1280] = np.arange(256, dtype=np.float32) - 127.0  # integer ramp: many round() ties
    d, qs, bs = hk.quantize_q8_k(torch.from_numpy(x).cuda(), k)
    d, qs, bs = d.cpu().numpy(), qs.cpu().numpy(), bs.cpu().numpy()
    for c in range(cols):
        rd, rq, rb = oracle.quantize_q8_k(x[c * k:(c + 1) * k])
        sl = slice(c * k, (c + 1) * k)
        assert np.array_equal(d[c * 8:(c + 1) * 8].view(np.uint32), rd.view(np.uint32))
        assert np.array_equal(qs[sl], rq)
        assert np.array_equal(bs[c * 64:(c + 1) * 64], rb)


def _oracle_matmul(oracle, type_id, w, x, k, rows, cols):
    s = oracle.prepare_scales(type_id, w, k, rows)
    return oracle.matmul_prepared(type_id, w, s, x, k, rows, cols, threads=oracle.cpu_threads())


@pytest.mark.parametrize("type_id,k,rows,cols", [
    (syn.Q4_K, 2048, 16384, 1),    # config 1
    (syn.Q4_K, 2048, 16384, 5),
    (syn.Q4_K, 2048, 2048, 8),
    (syn.Q4_K, 2048, 40, 3),       # ragged tile
    (syn.Q4_K, 256, 7, 1),         # one block per row
    (syn.Q4_K, 768, 100, 13),      # 3 blocks, > 8 columns
    (syn.Q6_K, 16384, 2048, 1),    # config 2 down projection (relay over a CTA pair)
    (syn.Q4_K, 16384, 2048, 1),
    (syn.Q4_K, 8192, 1000, 2),     # 32 blocks: two per warp over the pair, ragged tile
    (syn.Q6_K, 16384, 2048, 8),
    (syn.Q6_K, 2048, 520, 2),
    (syn.Q6_K, 512, 33, 9),
    # tensor-core GEMV (3..8 columns): persistent, in-CTA and cluster splits
    (syn.Q6_K, 16384, 2048, 5),    # verify-width down projection
    (syn.Q4_K, 256, 7, 3),         # one block, one ragged tile
    (syn.Q6_K, 768, 100, 6),
    (syn.Q4_K, 4096, 65, 7),
    # exact lane sums on the tensor cores (Q4_K, 2..8 columns, <= 16 blocks)
    (syn.Q4_K, 2048, 520, 2),
    (syn.Q4_K, 3840, 33, 6),       # 15 blocks, ragged tile
    (syn.Q4_K, 512, 4096, 4),
    # tensor-core path (>= 16 columns)
    (syn.Q4_K, 2048, 2048, 64),
    (syn.Q4_K, 768, 100, 70),      # ragged rows and columns
    (syn.Q4_K, 2048, 1024, 512),   # prefill width
    (syn.Q6_K, 2048, 520, 64),
    (syn.Q6_K, 16384, 2048, 16),
    (syn.Q6_K, 256, 33, 17),
])
@pytest.mark.parametrize("order", ["exact", "reordered"])
def test_matmul_matches_oracle(oracle, type_id, k, rows, cols, order):
    if order == "reordered" and cols >= 16:
        pytest.skip("16+ columns take the tensor-core path in either order")
    w = syn.quant_weight(type_id, rows, k, seed=rows * 3 + cols)
    x = syn.activations(cols, k, seed=cols + 100)
    h = hk.create_quantized_weight_handle(TNAME[type_id], w, k, rows)
    hk.set_matmul_order(order == "exact")
    try:
        got = hk.mat_mul_quantized_resident(h, torch.from_numpy(x).cuda(), k, rows, cols).cpu().numpy()
    finally:
        hk.set_matmul_order(True)
        hk.release_quantized_weight_handle(h)
    ref = _oracle_matmul(oracle, type_id, w, x, k, rows, cols)
    if order == "exact" and cols < 16:
        _bitwise(got, ref, "exact-order matmul")
        return
    mag = _magnitude(oracle, type_id, w, x, k, rows, cols)
    n_reassoc = _close(got, ref, mag, k // 256)
    print(f"outputs needing the re-association term: {n_reassoc} of {got.size}")


@pytest.mark.parametrize("cols", [1, 2, 4, 5, 8])
def test_multi_projection_config2(oracle, cols):
    k = 2048
    specs = [("Q", syn.Q4_K, 2048), ("K", syn.Q4_K, 512), ("V", syn.Q6_K, 512), ("gate", syn.Q4_K, 16384),
             ("up", syn.Q4_K, 16384)]
    x = syn.activations(cols, k, seed=5)
    ws = [syn.quant_weight(t, r, k, seed=50 + i) for i, (_, t, r) in enumerate(specs)]
    hs = [hk.create_quantized_weight_handle(TNAME[t], w, k, r) for (_, t, r), w in zip(specs, ws)]
    try:
        outs = hk.mat_mul_quantized_resident_multi(hs, torch.from_numpy(x).cuda(), k, cols)
        outs = [o.cpu().numpy() for o in outs]
    finally:
        for h in hs:
            hk.release_quantized_weight_handle(h)
    for (name, t, r), w, got in zip(specs, ws, outs):
        _bitwise(got, _oracle_matmul(oracle, t, w, x, k, r, cols), name)


@pytest.mark.parametrize("cols,residual", [(1, False), (1, True), (5, True), (8, True)])
def test_matmul_rmsnorm_matches_oracle(oracle, cols, residual):
    # hpc_matmul_rmsnorm_f32 (the step's norm-fused QKV / gate-up form) against
    # the oracle's rmsNorm rows -> quantize_q8_k -> prepared matmul, bit for bit
    from oracle import oracle as o
    k, eps = 2048, 1e-6
    specs = [(syn.Q4_K, 16384), (syn.Q6_K, 512)]
    g = np.random.default_rng(cols + 10 * residual)
    x = g.normal(0, 1, (cols, k)).astype(np.float32)
    y = g.normal(0, 3, (cols, k)).astype(np.float32)
    w_post = (1 + g.normal(0, 0.1, k)).astype(np.float32)
    w_pre = (1 + g.normal(0, 0.1, k)).astype(np.float32)
    ws = [syn.quant_weight(t, r, k, seed=70 + i) for i, (t, r) in enumerate(specs)]
    hs = [hk.create_quantized_weight_handle(TNAME[t], w, k, r) for (t, r), w in zip(specs, ws)]
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    try:
        outs, h_out = hk.mat_mul_rmsnorm(hs, dev(x), dev(w_pre), cols, y=dev(y) if residual else None,
                                         w_post=dev(w_post) if residual else None, eps=eps)
        outs = [t.cpu().numpy() for t in outs]
    finally:
        for h in hs:
            hk.release_quantized_weight_handle(h)
    h = (x + o.rms_norm_rows(y, w_post, eps)).astype(np.float32) if residual else x
    if residual:
        _bitwise(h_out.cpu().numpy().reshape(cols, k), h, "residual stream")
    n = o.rms_norm_rows(h, w_pre, eps)
    for (t, r), w, got in zip(specs, ws, outs):
        _bitwise(got, _oracle_matmul(oracle, t, w, n, k, r, cols), f"type {t} x {r}")


@pytest.mark.parametrize("rows,k,cols", [(256, 512, 64), (1000, 768, 70), (16384, 2048, 512), (32, 256, 16)])
def test_tcgen05_matmul_equals_mma_sync(rows, k, cols):
    # the tcgen05 kind::i8 matmul (split 3-bit scale halves, accumulators in
    # tensor memory) against the mma.sync one: the same integer block sums and
    # f32 combine, so the outputs are bit-identical (shapes whose mma.sync
    # launch does not split K)
    w = syn.quant_weight(syn.Q4_K, rows, k, seed=rows + cols)
    x = torch.from_numpy(syn.activations(cols, k, seed=cols + 3)).cuda()
    h = hk.create_quantized_weight_handle("Q4_K", w, k, rows)
    try:
        hk.set_wide_matmul_kind(0)
        ref = hk.mat_mul_quantized_resident(h, x, k, rows, cols).cpu().numpy()
        hk.set_wide_matmul_kind(1)
        got = hk.mat_mul_quantized_resident(h, x, k, rows, cols).cpu().numpy()
    finally:
        hk.set_wide_matmul_kind(0)
        hk.release_quantized_weight_handle(h)
    _bitwise(got, ref, "tcgen05 vs mma.sync")


def test_one_shot_host_api(oracle):
    k, rows, cols = 1024, 300, 3
    w = syn.quant_weight(syn.Q6_K, rows, k, seed=9)
    x = syn.activations(cols, k, seed=10)
    got = hk.mat_mul_quantized("Q6_K", w.tobytes(), x, k, rows, cols)
    _bitwise(got, oracle.matmul_quantized(syn.Q6_K, w, x, k, rows, cols), "one-shot matmul")


def test_zero_columns_and_errors():
    k, rows = 512, 10
    w = syn.quant_weight(syn.Q4_K, rows, k, seed=1)
    h = hk.create_quantized_weight_handle("Q4_K", w, k, rows)
    try:
        out = hk.mat_mul_quantized_resident(h, torch.empty(0, device="cuda"), k, rows, 0)
        assert out.numel() == 0
        with pytest.raises(hk.CudaKernelError, match="shape mismatch"):
            hk.mat_mul_quantized_resident(h, torch.zeros(k, device="cuda"), k, rows + 1, 1)
    finally:
        hk.release_quantized_weight_handle(h)
    with pytest.raises(hk.CudaKernelError, match="unsupported type"):
        hk.create_quantized_weight_handle("Q8_0", np.zeros(34, np.uint8), 32, 1)


def test_repeated_calls_are_deterministic():
    k, rows, cols = 16384, 256, 4
    w = syn.quant_weight(syn.Q6_K, rows, k, seed=2)
    x = torch.from_numpy(syn.activations(cols, k, seed=3)).cuda()
    h = hk.create_quantized_weight_handle("Q6_K", w, k, rows)
    try:
        a = hk.mat_mul_quantized_resident(h, x, k, rows, cols)
        b = hk.mat_mul_quantized_resident(h, x, k, rows, cols)
        assert torch.equal(a, b)
    finally:
        hk.release_quantized_weight_handle(h)


@pytest.mark.parametrize("type_id,k,rows,cols", [(syn.Q4_K, 2048, 512, 3), (syn.Q6_K, 2048, 300, 1),
                                                 (syn.Q6_K, 16384, 64, 2), (syn.Q4_K, 256, 33, 9)])
def test_matmul_dequantized_bit_exact(oracle, type_id, k, rows, cols):
    # hp_matmul_dequantized_f32 (lib.rs:103-154): bit-exact dequantized rows,
    # one sequential f32 chain per (row, column) -- equal to the oracle bit for
    # bit, through the one-shot host entry point and the resident one.
    w = syn.quant_weight(type_id, rows, k, seed=31 + rows)
    x = syn.activations(cols, k, seed=32 + cols)
    ref = oracle.matmul_dequantized(type_id, w, x, k, rows, cols)
    got = hk.mat_mul_dequantized(TNAME[type_id], w, x, k, rows, cols)
    assert np.array_equal(got.view(np.uint32), ref.astype(np.float32).view(np.uint32))
    h = hk.create_quantized_weight_handle(TNAME[type_id], w, k, rows)
    try:
        res = hk.mat_mul_dequantized_resident(h, torch.from_numpy(x).cuda(), k, rows, cols).cpu().numpy()
    finally:
        hk.release_quantized_weight_handle(h)
    assert np.array_equal(res.view(np.uint32), ref.astype(np.float32).view(np.uint32))
