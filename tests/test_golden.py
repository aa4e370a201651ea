"""Committed golden fixtures (tests/golden/kquant_golden.npz, made by
tests/golden/make_golden.py) checked against the oracle on CPU and against
the CUDA path through the C-ABI on the GPU.

Dequantization and Q8_K quantization are bit-exact on both sides; GEMV
outputs and LM-head values are within rtol 1e-3 / atol 1e-4 on the GPU
(exact on the CPU, where the oracle made them); top-k ids match exactly
(the fixture has no near-ties: checked below).
"""
import hashlib
from pathlib import Path

import numpy as np
import pytest

from heliopause_b200 import synthetic as syn

GOLD = Path(__file__).resolve().parent / "golden" / "kquant_golden.npz"
ROWS, K, COLS = 8, 512, 2
LM_ROWS, LM_K, LM_SEED, LM_TOP = 1024, 512, 104, 16


@pytest.fixture(scope="module")
def gold():
    with np.load(GOLD) as z:
        return {k: z[k] for k in z.files}


def _lm_weight(gold):
    w = syn.q6_k_weight(LM_ROWS, LM_K, seed=LM_SEED)
    assert hashlib.sha256(w.tobytes()).digest() == gold["lm_w_sha256"].tobytes(), "synthetic generator drifted"
    return w


# ----------------------------------------------------------------- CPU side --

@pytest.mark.parametrize("name,tid", [("q4k", syn.Q4_K), ("q6k", syn.Q6_K)])
def test_oracle_dequant_equals_gguf_fixture(oracle, gold, name, tid):
    got = oracle.dequantize(tid, gold[f"{name}_w"], K, ROWS)
    assert np.array_equal(got.view(np.uint32), gold[f"{name}_deq"].reshape(ROWS, K).view(np.uint32))


def test_oracle_q8_k_equals_fixture(oracle, gold):
    d, qs, bs = oracle.quantize_q8_k(gold["x"])
    assert np.array_equal(d.view(np.uint32), gold["q8_d"].view(np.uint32))
    assert np.array_equal(qs, gold["q8_qs"])
    assert np.array_equal(bs, gold["q8_bsums"])


@pytest.mark.parametrize("name,tid", [("q4k", syn.Q4_K), ("q6k", syn.Q6_K)])
def test_oracle_matmul_equals_fixture(oracle, gold, name, tid):
    w = gold[f"{name}_w"]
    got = oracle.matmul_prepared(tid, w, oracle.prepare_scales(tid, w, K, ROWS), gold["x"], K, ROWS, COLS)
    assert np.array_equal(got.view(np.uint32), gold[f"{name}_out"].view(np.uint32))


def test_oracle_topk_equals_fixture(oracle, gold):
    w = _lm_weight(gold)
    logits = oracle.matmul_prepared(syn.Q6_K, w, oracle.prepare_scales(syn.Q6_K, w, LM_K, LM_ROWS),
                                    gold["lm_hidden"], LM_K, LM_ROWS, COLS)
    for c in range(COLS):
        lc = logits[c * LM_ROWS:(c + 1) * LM_ROWS]
        ids, vals = oracle.topk(lc, LM_TOP)
        assert np.array_equal(ids, gold["lm_ids"][c]) and np.array_equal(vals, gold["lm_vals"][c])
        # the fixture's top-(k+1) has no near-ties, so GPU ids must match exactly
        srt = np.sort(lc)[::-1][:LM_TOP + 1].astype(np.float64)
        gaps = srt[:-1] - srt[1:]
        assert np.all(gaps > 1e-4 + 1e-3 * np.abs(srt[1:])), "fixture has a near-tie"


# ----------------------------------------------------------------- GPU side --

@pytest.fixture(scope="module")
def dev():
    import torch

    from heliopause_b200 import kernels as hk
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    hk.init_device(0)
    return hk, torch


def _within(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    assert np.all(np.abs(got - ref) <= 1e-4 + 1e-3 * np.abs(ref))


@pytest.mark.gpu
@pytest.mark.parametrize("name,tname", [("q4k", "Q4_K"), ("q6k", "Q6_K")])
def test_gpu_dequant_and_gemv_equal_fixture(gold, dev, name, tname):
    hk, torch = dev
    h = hk.create_quantized_weight_handle(tname, gold[f"{name}_w"], K, ROWS)
    try:
        deq = hk.dequantize_resident(h).cpu().numpy()
        out = hk.mat_mul_quantized_resident(h, torch.from_numpy(gold["x"]).cuda(), K, ROWS, COLS).cpu().numpy()
    finally:
        hk.release_quantized_weight_handle(h)
    assert np.array_equal(deq.reshape(-1).view(np.uint32), gold[f"{name}_deq"].reshape(-1).view(np.uint32))
    _within(out, gold[f"{name}_out"])


@pytest.mark.gpu
def test_gpu_q8_k_equals_fixture(gold, dev):
    hk, torch = dev
    d, qs, bs = hk.quantize_q8_k(torch.from_numpy(gold["x"]).cuda(), K)
    assert np.array_equal(d.cpu().numpy().view(np.uint32), gold["q8_d"].view(np.uint32))
    assert np.array_equal(qs.cpu().numpy(), gold["q8_qs"])
    assert np.array_equal(bs.cpu().numpy(), gold["q8_bsums"])


@pytest.mark.gpu
def test_gpu_lm_head_topk_equals_fixture(gold, dev):
    hk, torch = dev
    h = hk.create_quantized_weight_handle("Q6_K", _lm_weight(gold), LM_K, LM_ROWS)
    try:
        ids, vals = hk.lm_head_topk(h, torch.from_numpy(gold["lm_hidden"]).cuda(), COLS, LM_TOP)
    finally:
        hk.release_quantized_weight_handle(h)
    ids, vals = ids.cpu().numpy().reshape(COLS, LM_TOP), vals.cpu().numpy().reshape(COLS, LM_TOP)
    assert np.array_equal(ids, gold["lm_ids"])
    _within(vals, gold["lm_vals"])
