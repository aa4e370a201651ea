"""Generates the committed golden fixtures in this folder.

    python tests/golden/make_golden.py

kquant_golden.npz holds, for seeded BASELINE-distribution inputs small
enough to read:
  * q4k_w / q6k_w: GGUF-layout Q4_K / Q6_K weights (8 rows x 512) and
    q4k_deq / q6k_deq: their dequantization by gguf-py 0.19.0
    (gguf.quants.dequantize, an independent numpy restatement of the GGML
    block formats; the Heliopause tree has no K-quant known-answer test);
  * x: two f32 activation columns of 512 and q8_d / q8_qs / q8_bsums: their
    Q8_K quantization by the C oracle (quantize_q8_k, lib.rs:1774-1811);
  * q4k_out / q6k_out: the oracle's hp_matmul_quantized_prepared_f32
    (lib.rs:225-298) of each weight with x, out[col*rows + row];
  * lm_hidden / lm_ids / lm_vals: a 1024-row Q6_K head over 512 (not
    stored: regenerated from seed LM_SEED, its SHA-256 in lm_w_sha256) with
    two hidden columns and the oracle's top-16 per column (value desc, id
    asc; runtime.ts:514-527).
The oracle is itself pinned by tests/test_oracle_pins.py; these files freeze
its outputs so that a change to either side shows up as a fixture mismatch.
"""
from __future__ import annotations

import sys
from pathlib import Path

import hashlib

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from heliopause_b200 import synthetic as syn  # noqa: E402
from oracle import oracle  # noqa: E402

ROWS, K, COLS = 8, 512, 2
LM_ROWS, LM_K, LM_SEED = 1024, 512, 104


def main() -> None:
    import gguf

    out = {}
    for name, tid, qt in (("q4k", syn.Q4_K, "Q4_K"), ("q6k", syn.Q6_K, "Q6_K")):
        w = syn.quant_weight(tid, ROWS, K, seed=101 if tid == syn.Q4_K else 102)
        deq = gguf.quants.dequantize(w.reshape(ROWS, -1), getattr(gguf.GGMLQuantizationType, qt))
        out[f"{name}_w"] = w
        out[f"{name}_deq"] = deq.astype(np.float32)
    x = syn.activations(COLS, K, seed=103)
    d, qs, bs = oracle.quantize_q8_k(x)
    out["x"], out["q8_d"], out["q8_qs"], out["q8_bsums"] = x, d, qs, bs
    for name, tid in (("q4k", syn.Q4_K), ("q6k", syn.Q6_K)):
        w = out[f"{name}_w"]
        s = oracle.prepare_scales(tid, w, K, ROWS)
        out[f"{name}_out"] = oracle.matmul_prepared(tid, w, s, x, K, ROWS, COLS)
    lw = syn.q6_k_weight(LM_ROWS, LM_K, seed=LM_SEED)
    hid = syn.activations(COLS, LM_K, seed=108)  # first seed from 105 whose top-17 has no near-tie
    logits = oracle.matmul_prepared(syn.Q6_K, lw, oracle.prepare_scales(syn.Q6_K, lw, LM_K, LM_ROWS), hid, LM_K,
                                    LM_ROWS, COLS)
    ids, vals = zip(*(oracle.topk(logits[c * LM_ROWS:(c + 1) * LM_ROWS], 16) for c in range(COLS)))
    out["lm_w_sha256"] = np.frombuffer(hashlib.sha256(lw.tobytes()).digest(), np.uint8)
    out["lm_hidden"] = hid
    out["lm_ids"], out["lm_vals"] = np.stack(ids).astype(np.int32), np.stack(vals).astype(np.float32)
    np.savez_compressed(HERE / "kquant_golden.npz", **out)
    print("wrote", HERE / "kquant_golden.npz", sum(v.nbytes for v in out.values()), "bytes raw")


if __name__ == "__main__":
    main()
