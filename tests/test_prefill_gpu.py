"""Prefill (hpc_model_prefill) against the oracle decoder and the decode path.

  * parity: n hidden vectors at positions start..start+n-1 through every
    layer equal the oracle decoder's layer loop on the same input
    (oracle/decoder_oracle.py `layer`, the WASM provider's forward for n
    positions with the causal mask), at n = 40 (tensor-core matmuls), n = 7
    (GEMV), n = 200 over a 256-token context (the attention's key window
    split in two), n = 60 after a 100-token prefix already in the cache, and
    n = 40 with 8 query heads per KV head (the unsplit attention form).
    K/V cache rows of the first KV layer: within 1e-3 (|ref| + rms(ref)).
    Final residual: every token within 3e-2, and at least 90% of tokens
    within 1e-3 of that scale; K/V rows of deeper layers the same with 6e-2.
    The reference algorithm is discontinuous -- Q8_K rounding of every
    matmul input and the f16 casts of the attention output and GEGLU -- and
    the oracle itself moves single tokens when its input is perturbed by 1e-7
    relative: by up to ~3e-3 of that scale on the one-layer form of the
    40-token case, and by up to 1.79e-2 (4-5% of the tokens beyond 1e-3) on
    the 3-layer 200-token case, whose flips compound through the later
    tokens' attention (its layer-1 K/V rows move by up to 3.1e-2; layer 0's
    by 4.5e-7).  A different but equally exact summation order flips
    the same steps;
  * consistency: prefilling a prompt's embedded tokens leaves the same KV
    cache and the same next-token top-k as running the prompt through the
    batched forward in 8-token steps.
"""
from dataclasses import replace

import numpy as np
import pytest
import torch

from heliopause_b200 import kernels as hk
from heliopause_b200.model import CudaDecoderModel, DecoderShape, SyntheticWeights

pytestmark = pytest.mark.gpu

SHAPE = DecoderShape(hidden=2048, heads=8, kv_heads=2, head_dim=256, ffn=2048, vocab=4096, layers=3, kv_layers=2,
                     context=128)


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    hk.init_device(0)


def _close(got, ref, what):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.sqrt(np.mean(ref ** 2))
    err = np.abs(got - ref)
    assert np.all(err <= 1e-3 * (np.abs(ref) + scale)), f"{what}: max err {err.max():.3g} (scale {scale:.3g})"


def _close_tokens(got, ref, what, bound=3e-2, within=0.9):
    """Per-token bound with room for single rounding-step flips (see above)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rel = np.abs(got - ref) / (np.abs(ref) + np.sqrt(np.mean(ref ** 2)))
    worst = rel.max(axis=1)
    print(f"{what}: per-token max relative error x1e3", np.round(worst * 1e3, 3).tolist())
    assert worst.max() <= bound, f"{what}: token {int(worst.argmax())} off by {worst.max():.3g}"
    assert (worst <= 1e-3).mean() >= within, f"{what}: {(worst > 1e-3).sum()} of {len(worst)} tokens beyond 1e-3"


@pytest.mark.parametrize("n,context,start,kv_heads", [(40, 128, 0, 2), (7, 128, 0, 2),
                                                      (200, 256, 0, 2),    # two 128-key splits per late query tile
                                                      (60, 256, 100, 2),   # continuing after a 100-token prefix
                                                      (40, 128, 0, 1)])    # 8 query heads per KV head: unsplit form
def test_prefill_matches_oracle(n, context, start, kv_heads):
    from oracle.decoder_oracle import OracleDecoder
    shape = replace(SHAPE, context=context, kv_heads=kv_heads)
    nkv = shape.kv_heads
    w = SyntheticWeights(shape, seed=21)
    gpu = CudaDecoderModel(shape, max_tokens=8, top_k=64)
    try:
        gpu.load_synthetic(w)
        ref = OracleDecoder(shape, w)
        g = np.random.default_rng(n + start)
        for kl in range(shape.kv_layers):
            kc = np.zeros((context, nkv, 256), np.float32)
            vc = np.zeros((256, nkv, context), np.float32)
            if start:  # an existing prefix in the cache
                kc[:start] = g.standard_normal((start, nkv, 256))
                vc[:, :, :start] = g.standard_normal((256, nkv, start))
            ref.set_kv(kl, kc.copy(), vc.copy())
            gk, gv = gpu.kv(kl)
            gk.copy_(torch.from_numpy(kc))
            gv.copy_(torch.from_numpy(vc))
        x = g.standard_normal((n, shape.hidden)).astype(np.float32)
        got = gpu.prefill(torch.from_numpy(x), start).cpu().numpy()
        h = x.reshape(-1)
        for layer in range(shape.layers):
            h = ref.layer(layer, h, list(range(start, start + n)))
        # after the random prefix the oracle itself moves single tokens by up
        # to 3.96e-2 (15-18% beyond 1e-3) under a 1e-7 input perturbation
        bound, within = (6e-2, 0.8) if start else (3e-2, 0.9)
        _close_tokens(got, h.reshape(n, -1), "final residual", bound, within)
        t = start + n
        for kl in range(shape.kv_layers):
            gk, gv = gpu.kv(kl)
            rk, rv = ref.kv[kl]
            gk, gv = gk[:t].cpu().numpy(), gv[:, :, :t].cpu().numpy()
            if kl == 0:  # computed from the input alone: no upstream flips
                _close(gk, rk[:t], f"K layer {kl}")
                _close(gv, rv[:, :, :t], f"V layer {kl}")
            else:  # rows of deeper layers inherit the earlier layers' flips
                _close_tokens(gk.reshape(t, -1), rk[:t].reshape(t, -1), f"K layer {kl}", 6e-2, within)
                _close_tokens(gv.transpose(2, 1, 0).reshape(t, -1), rv[:, :, :t].transpose(2, 1, 0).reshape(t, -1),
                              f"V layer {kl}", 6e-2, within)
    finally:
        gpu.close()


def test_prefill_equals_batched_forward():
    w = SyntheticWeights(SHAPE, seed=22)
    n = 24
    ids = [int(t) for t in np.random.default_rng(5).integers(0, SHAPE.vocab, n)]
    a = CudaDecoderModel(SHAPE, max_tokens=8, top_k=64)
    b = CudaDecoderModel(SHAPE, max_tokens=8, top_k=64)
    try:
        a.load_synthetic(w)
        b.load_synthetic(w)
        # embedding rows * sqrt(D) (prepareInput, layers.ts:54-67), as the embed kernel computes them
        emb = hk.dequantize_resident(a.lm_head_handle)[torch.tensor(ids, device="cuda")]
        hidden = (emb.double() * np.sqrt(SHAPE.hidden)).float()
        ha = a.prefill(hidden, 0)
        for s in range(0, n, 8):
            _, _, hb = b.forward(ids[s:s + 8], list(range(s, s + 8)), 8, return_hidden=True)
        _close_tokens(ha[-8:].cpu().numpy(), hb.cpu().numpy(), "last 8 residuals")
        for kl in range(SHAPE.kv_layers):
            _close(a.kv(kl)[0][:n].cpu().numpy(), b.kv(kl)[0][:n].cpu().numpy(), f"K layer {kl}")
            _close(a.kv(kl)[1][:, :, :n].cpu().numpy(), b.kv(kl)[1][:, :, :n].cpu().numpy(), f"V layer {kl}")
        ia, va = a.decode_token(77, n, 16)
        ib, vb = b.decode_token(77, n, 16)
        assert torch.allclose(va, vb, rtol=1e-3, atol=1e-3)
        assert ia[0].item() == ib[0].item() or abs(va[0].item() - va[1].item()) < 1e-2
    finally:
        a.close()
        b.close()


def test_prefill_rejects_bad_sizes():
    gpu = CudaDecoderModel(replace(SHAPE, context=64), max_tokens=8, top_k=64)
    try:
        gpu.load_synthetic(SyntheticWeights(replace(SHAPE, context=64), seed=1))
        with pytest.raises(hk.CudaKernelError):
            gpu.prefill(torch.zeros(65, SHAPE.hidden), 0)
    finally:
        gpu.close()
