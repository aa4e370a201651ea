"""Seeded synthetic GGUF-format weights and activations.

The reference quotes no public dataset for this path; every configuration is
defined by shapes and value distributions, so seeded inputs with exactly those
distributions stand in for real model files.  Generator: numpy PCG64.

Block formats follow packages/engine/wasm-kernels/src/lib.rs (Q4_K: 144-byte
blocks, lib.rs:1630-1664; Q6_K: 210-byte blocks, lib.rs:1709-1744).
"""
from __future__ import annotations

import numpy as np

QK = 256
Q4_K, Q5_K, Q6_K, IQ4_XS, Q8_0, Q4_0 = 1, 2, 3, 4, 5, 6
BLOCK = {Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210), IQ4_XS: (256, 136), Q8_0: (32, 34), Q4_0: (32, 18)}


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def row_bytes(type_id: int, k: int) -> int:
    blk, nbytes = BLOCK[type_id]
    if k % blk:
        raise ValueError(f"K={k} is not a multiple of {blk}")
    return k // blk * nbytes


def pack_scale_min_k4(sc: np.ndarray, mn: np.ndarray) -> np.ndarray:
    """Inverse of get_scale_min_k4 (lib.rs:2250-2259): 8 six-bit scales and 8
    six-bit mins -> 12 bytes.  sc, mn: uint8 [..., 8] in 0..63."""
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    out = np.empty(sc.shape[:-1] + (12,), np.uint8)
    out[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    out[..., 4:8] = (mn[..., 0:4] & 63) | ((mn[..., 4:8] >> 4) << 6)
    out[..., 8:12] = (sc[..., 4:8] & 15) | ((mn[..., 4:8] & 15) << 4)
    return out


def _f16_bytes(values: np.ndarray) -> np.ndarray:
    return values.astype(np.float16).view(np.uint8).reshape(values.shape + (2,))


def q4_k_weight(rows: int, k: int, seed: int) -> np.ndarray:
    """GGUF Q4_K rows: d = f16(|N(0,1)|*0.01), dmin = f16(|N(0,1)|*0.005),
    8 scales + 8 mins uniform 0..63, qs bytes uniform 0..255."""
    g = rng(seed)
    nb = rows * (k // QK)
    blocks = np.empty((nb, 144), np.uint8)
    blocks[:, 0:2] = _f16_bytes(np.abs(g.standard_normal(nb, dtype=np.float32)) * np.float32(0.01))
    blocks[:, 2:4] = _f16_bytes(np.abs(g.standard_normal(nb, dtype=np.float32)) * np.float32(0.005))
    sc = g.integers(0, 64, size=(nb, 8), dtype=np.uint8)
    mn = g.integers(0, 64, size=(nb, 8), dtype=np.uint8)
    blocks[:, 4:16] = pack_scale_min_k4(sc, mn)
    blocks[:, 16:144] = g.integers(0, 256, size=(nb, 128), dtype=np.uint8)
    return blocks.reshape(-1)


def q6_k_weight(rows: int, k: int, seed: int) -> np.ndarray:
    """GGUF Q6_K rows: ql, qh and the 16 int8 scales uniform over their full
    byte range; d = f16(|N(0,1)|*0.01) (finite, no Inf/NaN halves)."""
    g = rng(seed)
    nb = rows * (k // QK)
    blocks = np.empty((nb, 210), np.uint8)
    blocks[:, 0:208] = g.integers(0, 256, size=(nb, 208), dtype=np.uint8)
    blocks[:, 208:210] = _f16_bytes(np.abs(g.standard_normal(nb, dtype=np.float32)) * np.float32(0.01))
    return blocks.reshape(-1)


def quant_weight(type_id: int, rows: int, k: int, seed: int) -> np.ndarray:
    if type_id == Q4_K:
        return q4_k_weight(rows, k, seed)
    if type_id == Q6_K:
        return q6_k_weight(rows, k, seed)
    raise ValueError(f"no synthetic generator for type {type_id}")


def activations(cols: int, k: int, seed: int) -> np.ndarray:
    """fp32 ~N(0,1), column-major by activation column: x[col*K + i]."""
    return rng(seed).standard_normal(cols * k, dtype=np.float32)
