"""Pins the CPU oracle to the reference's own known-answer tests.

Each case cites the reference test it restates (paths inside the Heliopause
tree).  K-quant dequantization is additionally cross-checked bit for bit
against gguf-py 0.19.0 (an independent numpy implementation of the GGML block
formats).  Runs on CPU.
"""
import math
import struct

import numpy as np
import pytest

from heliopause_b200 import synthetic as syn


def test_f16_known_values(oracle):
    # packages/engine/test/quant.test.ts:12-17
    assert oracle.f16_to_f32(0x0000) == 0.0
    assert oracle.f16_to_f32(0x3C00) == 1.0
    assert oracle.f16_to_f32(0xC000) == -2.0
    assert oracle.f16_to_f32(0x7C00) == math.inf


def test_f32_to_f16_ties(oracle):
    # quant.test.ts:19-22: the TS codec rounds ties to even ...
    assert oracle.f32_to_f16_ts(1 + 0.5 / 1024) == 0x3C00
    assert oracle.f32_to_f16_ts(1 + 1.5 / 1024) == 0x3C02
    # ... while the Rust codec (lib.rs:2558) rounds the dropped half up.
    assert oracle.f32_to_f16_rust(1 + 0.5 / 1024) == 0x3C01
    assert oracle.f32_to_f16_rust(1 + 1.5 / 1024) == 0x3C02


def test_f32_to_f16_ts_matches_numpy_away_from_clamp(oracle):
    # numpy's cast is IEEE round-to-nearest-even; the TS codec agrees except
    # that it clamps |x| >= 65504 to 0x7bff instead of overflowing and
    # flushes |x| < 2^-24 to zero (quant.ts:652-654).
    g = np.random.default_rng(5)
    vals = np.concatenate([g.standard_normal(2000).astype(np.float32) * s for s in (1e-6, 1e-3, 1.0, 100.0)])
    vals = vals[np.abs(vals) >= 2.0 ** -24]
    for v in vals:
        assert oracle.f32_to_f16_ts(float(v)) == int(np.float32(v).astype(np.float16).view(np.uint16))
    assert oracle.f32_to_f16_ts(70000.0) == 0x7BFF
    assert oracle.f32_to_f16_rust(70000.0) == 0x7BFF
    assert oracle.f32_to_f16_ts(4e-8) == 0x0000


def test_q8_0_dequant_block(oracle):
    # quant.test.ts:24-38
    b = bytearray(34)
    struct.pack_into("<H", b, 0, 0x3C00)
    for i in range(32):
        b[2 + i] = i if i < 16 else 256 - (i - 15)
    v = oracle.dequantize(oracle.Q8_0, b, 32)[0]
    assert (v[0], v[15], v[16], v[31]) == (0, 15, -1, -16)


def test_q4_0_dequant_block(oracle):
    # quant.test.ts:40-56
    b = bytearray(18)
    struct.pack_into("<H", b, 0, 0x4000)
    for i in range(16):
        b[2 + i] = (i & 0x0F) | ((15 - i) << 4)
    v = oracle.dequantize(oracle.Q4_0, b, 32)[0]
    assert (v[0], v[7], v[8], v[15], v[16], v[31]) == (-16, -2, 0, 14, 14, -16)


def test_block_byte_sizes(oracle):
    # quant.test.ts:58-66
    assert oracle.row_bytes(oracle.Q4_0, 32) == 18
    assert oracle.row_bytes(oracle.Q8_0, 32) == 34
    assert oracle.row_bytes(oracle.Q4_K, 256) == 144
    assert oracle.row_bytes(oracle.Q5_K, 256) == 176
    assert oracle.row_bytes(oracle.Q6_K, 256) == 210
    assert oracle.row_bytes(oracle.IQ4_XS, 256) == 136


# --- q4-0-matmul.test.ts:20-82 fixture and its TS-mirror expectation ---------

def _q4_0_weight(rows, seed=1):
    # q4-0-matmul.test.ts:111-124
    import numpy as np
    out = bytearray(rows * 18)
    for r in range(rows):
        o = r * 18
        h = int(np.float32(0.125 * (r + seed)).astype(np.float16).view(np.uint16))
        struct.pack_into("<H", out, o, h)
        for i in range(16):
            lo = (r + i + seed) % 16
            hi = (r + 15 - i + seed) % 16
            out[o + 2 + i] = lo | (hi << 4)
    return bytes(out)


def _ts_quantize_q8_0(x, oracle):
    # quant.ts:483-507 (f64 arithmetic, Math.round = floor(v + 0.5), Int8Array wrap)
    d, qs = [], []
    for b in range(len(x) // 32):
        blk = [float(v) for v in x[b * 32:(b + 1) * 32]]
        amax = max(abs(v) for v in blk)
        scale = oracle.f16_to_f32(oracle.f32_to_f16_ts(amax / 127))
        inv = 1 / scale if scale else 0
        d.append(scale)
        for v in blk:
            q = math.floor(v * inv + 0.5)
            qs.append(((q + 128) % 256) - 128)
    return d, qs


def _ts_vec_dot_q4_0(row, d, qs, oracle):
    # quant.ts:529-549
    s = 0.0
    for b in range(len(d)):
        o = b * 18
        dd = oracle.f16_to_f32(row[o] | (row[o + 1] << 8)) * d[b]
        isum = 0
        for i in range(16):
            p = row[o + 2 + i]
            isum += ((p & 15) - 8) * qs[b * 32 + i] + ((p >> 4) - 8) * qs[b * 32 + i + 16]
        s += isum * dd
    return s


def test_q4_0_matmul_fixture_matches_ts_mirror(oracle):
    k, rows, cols = 32, 4, 2
    x = np.array([((i % 9) - 4) * 0.25 for i in range(k * cols)], np.float32)  # :126-132
    for seed in (1, 2):
        w = _q4_0_weight(rows, seed)
        expected = []
        for c in range(cols):
            d, qs = _ts_quantize_q8_0(x[c * k:(c + 1) * k], oracle)
            expected += [_ts_vec_dot_q4_0(w[r * 18:(r + 1) * 18], d, qs, oracle) for r in range(rows)]
        direct = oracle.matmul_quantized(oracle.Q4_0, w, x, k, rows, cols)
        scales = oracle.prepare_scales(oracle.Q4_0, w, k, rows)
        prepared = oracle.matmul_prepared(oracle.Q4_0, w, scales, x, k, rows, cols)
        threaded = oracle.matmul_prepared(oracle.Q4_0, w, scales, x, k, rows, cols, threads=2)
        for got in (direct, prepared, threaded):
            assert np.all(np.abs(got - np.array(expected)) < 1e-5)  # :145-150 tolerance


# --- K-quant dequantization against gguf-py --------------------------------

@pytest.mark.parametrize("type_id,qtype", [(syn.Q4_K, "Q4_K"), (syn.Q6_K, "Q6_K")])
def test_kquant_dequant_bit_exact_vs_gguf(oracle, type_id, qtype):
    import gguf
    rows, k = 16, 1024
    w = syn.quant_weight(type_id, rows, k, seed=21)
    ours = oracle.dequantize(type_id, w, k, rows)
    theirs = gguf.quants.dequantize(w.reshape(rows, -1), getattr(gguf.GGMLQuantizationType, qtype))
    assert theirs.shape == (rows, k)
    assert np.array_equal(ours.view(np.uint32), theirs.astype(np.float32).view(np.uint32))


def test_q8_k_quantize_rules(oracle):
    # lib.rs:1774-1811: first strictly larger |x| wins (keeping its sign);
    # an all-zero block gives d = 0 and q = 0.
    x = np.zeros(512, np.float32)
    x[3], x[7], x[10] = 2.0, -2.0, 1.0   # tie at |2|: index 3 (positive) wins
    x[256 + 5] = -3.0
    d, qs, bs = oracle.quantize_q8_k(x)
    assert d[0] == np.float32(1.0) / (np.float32(-127.0) / np.float32(2.0))
    assert qs[3] == -127 and qs[7] == 127 and qs[10] == -64
    assert bs[0] == -127 + 127 - 64 + 0
    assert d[1] == np.float32(1.0) / (np.float32(-127.0) / np.float32(-3.0)) and qs[256 + 5] == -127
    d2, q2, b2 = oracle.quantize_q8_k(np.zeros(256, np.float32))
    assert d2[0] == 0 and not q2.any() and not b2.any()


def test_kquant_dot_equals_dequant_reference(oracle):
    # Self-consistency: the integer block dot equals the f64 dot of the
    # dequantized weight row with the dequantized Q8_K activation.
    k = 2048
    x = syn.activations(1, k, seed=3)
    d, qs, _ = oracle.quantize_q8_k(x)
    xa = (qs.astype(np.float64).reshape(-1, 256) * d.astype(np.float64)[:, None]).reshape(-1)
    for t in (syn.Q4_K, syn.Q6_K):
        w = syn.quant_weight(t, 8, k, seed=4)
        got = oracle.matmul_quantized(t, w, x, k, 8, 1)
        wd = oracle.dequantize(t, w, k, 8).astype(np.float64)
        ref = wd @ xa
        mag = np.abs(wd) @ np.abs(xa)  # f32 rounding error scales with sum |w*x|
        assert np.all(np.abs(got - ref) <= 1e-6 * mag + 1e-6)


def test_prepared_and_multi_equal_direct(oracle):
    k, cols = 512, 3
    x = syn.activations(cols, k, seed=8)
    wa = syn.quant_weight(syn.Q4_K, 40, k, seed=9)
    wb = syn.quant_weight(syn.Q6_K, 24, k, seed=10)
    da = oracle.matmul_quantized(syn.Q4_K, wa, x, k, 40, cols)
    db = oracle.matmul_quantized(syn.Q6_K, wb, x, k, 24, cols)
    sa = oracle.prepare_scales(syn.Q4_K, wa, k, 40)
    sb = oracle.prepare_scales(syn.Q6_K, wb, k, 24)
    assert np.array_equal(oracle.matmul_prepared(syn.Q4_K, wa, sa, x, k, 40, cols), da)
    assert np.array_equal(oracle.matmul_prepared(syn.Q6_K, wb, sb, x, k, 24, cols, threads=3), db)
    ma, mb = oracle.matmul_multi([(syn.Q4_K, wa, sa, 40), (syn.Q6_K, wb, sb, 24)], x, k, cols)
    assert np.array_equal(ma, da) and np.array_equal(mb, db)


def test_driver_error_codes(oracle):
    w = syn.quant_weight(syn.Q4_K, 2, 256, seed=1)
    x = np.zeros(256, np.float32)
    with pytest.raises(oracle.OracleError) as e:
        oracle.matmul_quantized(syn.Q4_K, w, x, 256, 3, 1)  # weight length != rows*row_bytes
    assert e.value.code == oracle.ERR_SHAPE
    with pytest.raises(oracle.OracleError) as e:
        oracle.matmul_quantized(99, w, x, 256, 2, 1)
    assert e.value.code == oracle.ERR_TYPE
    with pytest.raises(oracle.OracleError) as e:
        oracle.matmul_quantized(syn.Q4_K, w, x, 200, 2, 1)  # K not a multiple of 256 (input_len check first)
    assert e.value.code == oracle.ERR_SHAPE


def test_split_rows(oracle):
    # thread-pool.ts:410-424
    assert oracle.split_rows(10, 4) == [(0, 3), (3, 3), (6, 2), (8, 2)]
    assert oracle.split_rows(2, 4) == [(0, 1), (1, 1)]


def test_topk_tie_rule(oracle):
    # runtime.ts:514-527: value descending, lower id first on ties.
    ids, vals = oracle.topk(np.array([1, 3, 3, 2, 3, 0], np.float32), 3)
    assert ids.tolist() == [1, 2, 4] and vals.tolist() == [3, 3, 3]
    ids, _ = oracle.topk(np.array([5, 1, 5, 7], np.float32), 2)
    assert ids.tolist() == [3, 0]


def test_synthetic_forward_top2(oracle):
    # forward-graph.test.ts:281-316: F32 token_embd [4,8], output_norm ones,
    # output.weight [4,3]; token 2 -> top ids [1, 0] with fixed values.
    seq = np.array([((i % 7) - 3) * 0.1 for i in range(32)], np.float32)
    emb = oracle.scale_embedding(seq[8:12], 4)
    norm = oracle.rms_norm_rows(emb, np.ones(4, np.float32), 1e-6)
    w = np.array([0.2, 0.1, -0.1, 0.3, -0.4, 0.2, 0.5, 0.1, 0.3, -0.2, 0.4, -0.3], np.float32).reshape(3, 4)
    logits = np.zeros(3, np.float32)
    for r in range(3):  # layers.ts:724-745 matMulDenseRows: sequential fround sum
        s = np.float32(0)
        for i in range(4):
            s = np.float32(s + np.float32(w[r, i] * norm[i]))
        logits[r] = s
    ids, vals = oracle.topk(logits, 2)
    assert ids.tolist() == [1, 0]
    assert np.allclose(vals, [0.5715285539627075, -0.16329389810562134], atol=2e-5)


def test_gqa_attention_small(oracle):
    # Attention over a 3-slot ring vs a direct f64 computation.
    head, nq, nkv, cap = 4, 2, 1, 3
    g = np.random.default_rng(0)
    q = g.standard_normal(nq * head).astype(np.float32)
    k = g.standard_normal(cap * nkv * head).astype(np.float32)
    v = g.standard_normal(cap * nkv * head).astype(np.float32)
    out = oracle.gqa_attention(q, k, v, head=head, nq=nq, nkv=nkv, ntok=1, nkvtok=3, kvstart=0, cap=cap,
                               scale=1.0, value_layout=0, qf16=False)
    kk = k.reshape(cap, head).astype(np.float64)
    vv = v.reshape(cap, head).astype(np.float64)
    for h in range(nq):
        s = kk @ q[h * head:(h + 1) * head].astype(np.float64)
        p = np.exp(s - s.max())
        p /= p.sum()
        assert np.allclose(out[h * head:(h + 1) * head], p @ vv, rtol=1e-5, atol=1e-6)
