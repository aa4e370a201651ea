"""GPU parity of the fused LM head + top-k against the oracle.

The oracle materializes every logit with the C restatement of lib.rs and
selects with the restated topK (runtime.ts:514-527).
  * default (reference) order, fewer than 16 columns: ids equal the oracle's
    (sets and order) and values equal bit for bit;
  * the reordered kernels (hpc_set_matmul_order(0)) and the tensor-core path
    (16+ columns): ids must match exactly, except that two oracle logits that
    differ by less than the matmul tolerance (|d| <= 1e-4 + 1e-3 |v|) may
    swap; values within the same tolerance.
"""
import numpy as np
import pytest
import torch

from heliopause_b200 import kernels as hk
from heliopause_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    hk.init_device(0)


def _tol(v):
    return 1e-4 + 1e-3 * np.abs(v)


def _check_topk(ids, vals, logits, k):
    ref_ids, ref_vals = None, None
    from oracle import oracle
    ref_ids, ref_vals = oracle.topk(logits, k)
    assert np.all(np.abs(vals - ref_vals) <= _tol(ref_vals)), "values outside tolerance"
    if not np.array_equal(ids, ref_ids):
        # allow swaps only between near-tied logits
        for i in np.nonzero(ids != ref_ids)[0]:
            a, b = logits[ids[i]], logits[ref_ids[i]]
            assert abs(a - b) <= _tol(b), f"rank {i}: id {ids[i]} vs {ref_ids[i]} not a near-tie"
        # membership may differ only at the boundary, again by a near-tie
        extra = set(ids.tolist()) ^ set(ref_ids.tolist())
        for e in extra:
            assert abs(logits[e] - ref_vals[-1]) <= _tol(ref_vals[-1])


@pytest.mark.parametrize("type_id,rows,k,cols", [
    (syn.Q6_K, 262144, 40, 1),   # config 3 LM head
    (syn.Q6_K, 262144, 40, 5),   # verify width
    (syn.Q6_K, 50000, 64, 3),    # ragged last tile, TOPK_MAX
    (syn.Q4_K, 4096, 1, 9),      # greedy (top-1), > 8 columns
    (syn.Q6_K, 40, 40, 1),       # k == rows
    # tensor-core LM head + top-k (3..8 columns)
    (syn.Q4_K, 4096, 64, 8),
    (syn.Q6_K, 100, 10, 4),      # fewer tiles than one CTA's warps
    # tensor-core path (>= 16 columns): materialized logits, chunked lists
    (syn.Q6_K, 20000, 40, 64),   # config-5 width, ragged last chunk
    (syn.Q6_K, 50000, 64, 17),
    (syn.Q4_K, 4096, 1, 20),
])
@pytest.mark.parametrize("order", ["exact", "reordered"])
def test_lm_head_topk_matches_oracle(oracle, type_id, rows, k, cols, order):
    if order == "reordered" and cols >= 16:
        pytest.skip("16+ columns take the tensor-core path in either order")
    kdim = 2048
    w = syn.quant_weight(type_id, rows, kdim, seed=rows + k)
    x = syn.activations(cols, kdim, seed=cols)
    name = "Q6_K" if type_id == syn.Q6_K else "Q4_K"
    h = hk.create_quantized_weight_handle(name, w, kdim, rows)
    hk.set_matmul_order(order == "exact")
    try:
        ids, vals = hk.lm_head_topk(h, torch.from_numpy(x).cuda(), cols, k)
        ids, vals = ids.cpu().numpy(), vals.cpu().numpy()
    finally:
        hk.set_matmul_order(True)
        hk.release_quantized_weight_handle(h)
    s = oracle.prepare_scales(type_id, w, kdim, rows)
    logits = oracle.matmul_prepared(type_id, w, s, x, kdim, rows, cols, threads=oracle.cpu_threads())
    for c in range(cols):
        lc = logits[c * rows:(c + 1) * rows]
        if order == "exact" and cols < 16:
            ref_ids, ref_vals = oracle.topk(lc, k)
            assert np.array_equal(ids[c], ref_ids), f"column {c}: ids differ"
            assert np.array_equal(vals[c].view(np.uint32), ref_vals.astype(np.float32).view(np.uint32))
        else:
            _check_topk(ids[c], vals[c], lc, k)


def test_ties_prefer_lower_id_and_softcap(oracle):
    # Identical rows give identical logits: the lower id must win every tie.
    kdim, rows = 256, 96
    one = syn.quant_weight(syn.Q6_K, 1, kdim, seed=3)
    w = np.tile(one, rows)
    x = syn.activations(1, kdim, seed=4)
    h = hk.create_quantized_weight_handle("Q6_K", w, kdim, rows)
    try:
        ids, vals = hk.lm_head_topk(h, torch.from_numpy(x).cuda(), 1, 10, id_offset=1000)
        ids2, vals2 = hk.lm_head_topk(h, torch.from_numpy(x).cuda(), 1, 10, softcap=30.0)
    finally:
        hk.release_quantized_weight_handle(h)
    assert ids.cpu().numpy()[0].tolist() == list(range(1000, 1010))
    v = vals.cpu().numpy()[0]
    assert np.all(v == v[0])
    capped = np.float32(np.tanh(np.float64(v[0]) / 30.0) * 30.0)
    assert np.all(vals2.cpu().numpy()[0] == capped)
    # the same on the tensor-core path: 16 columns, rows spread over chunks
    rows = 5000
    w = np.tile(one, rows)
    x = np.tile(syn.activations(1, kdim, seed=4), 16)
    h = hk.create_quantized_weight_handle("Q6_K", w, kdim, rows)
    try:
        ids, vals = hk.lm_head_topk(h, torch.from_numpy(x).cuda(), 16, 10, id_offset=7)
    finally:
        hk.release_quantized_weight_handle(h)
    assert all(r == list(range(7, 17)) for r in ids.cpu().numpy().tolist())
    tv = vals.cpu().numpy()
    assert np.all(tv == tv[0, 0]) and abs(tv[0, 0] - v[0]) <= _tol(v[0])
    # and at 3..8 columns, on the exact-order logits and on the tensor-core
    # LM head of the reordered kernels
    x = np.tile(syn.activations(1, kdim, seed=4), 5)
    h = hk.create_quantized_weight_handle("Q6_K", w, kdim, rows)
    try:
        for exact in (True, False):
            hk.set_matmul_order(exact)
            ids, vals = hk.lm_head_topk(h, torch.from_numpy(x).cuda(), 5, 10, id_offset=3)
            assert all(r == list(range(3, 13)) for r in ids.cpu().numpy().tolist())
            mv = vals.cpu().numpy()
            assert np.all(mv == mv[0, 0])
            assert (mv[0, 0] == v[0]) if exact else abs(mv[0, 0] - v[0]) <= _tol(v[0])
    finally:
        hk.set_matmul_order(True)
        hk.release_quantized_weight_handle(h)


def test_topk_errors():
    w = syn.quant_weight(syn.Q6_K, 8, 256, seed=1)
    h = hk.create_quantized_weight_handle("Q6_K", w, 256, 8)
    try:
        with pytest.raises(hk.CudaKernelError, match="shape mismatch"):
            hk.lm_head_topk(h, torch.zeros(256, device="cuda"), 1, 9)   # k > rows
        with pytest.raises(hk.CudaKernelError, match="shape mismatch"):
            hk.lm_head_topk(h, torch.zeros(256, device="cuda"), 1, 0)
    finally:
        hk.release_quantized_weight_handle(h)
    hk.device_error()  # no bounded wait timed out during the suite
