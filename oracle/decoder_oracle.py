"""CPU restatement of the WASM provider's decoder forward (parity oracle).

TEST INFRASTRUCTURE ONLY (see oracle.py).  Follows, step for step,
packages/engine/src/runner/wasm/layers.ts:
  prepareInput            :54-67     embedding row * sqrt(D)
  forwardAttentionLayer   :161-377   norms, q/k/v projections, RoPE, KV write,
                                     causal GQA attention (lib.rs:539-654) on the
                                     compacted range, f16 cast, o projection,
                                     post-attention norm + residual
  forwardFfn              :418-473   FFN norm, gate/up, GEGLU, down,
                                     post-FFN norm + residual
  forwardOutput           :381-416   output norm, LM head logits, softcap, topK
with every matmul through the restated quantized-prepared driver (the
reference's matMulKQ8K path, lib.rs:225-298).  All layers are full-attention;
layers >= kv_layers read the KV of layer kv_layers-1 (model.ts:382-388).
Returns per-position top-k (the WebGPU verify runner's per-position output,
webgpu/segment-runner.ts:1441-1450) plus the final residual stream.
"""
from __future__ import annotations

import numpy as np

from . import oracle as o


def causal_mask(positions, start: int, count: int) -> np.ndarray:
    """layers.ts:913-924."""
    pos = np.asarray(positions, np.int64)
    key = start + np.arange(count)
    return np.where(key[None, :] <= pos[:, None], 0.0, -np.inf).astype(np.float32).reshape(-1)


class OracleDecoder:
    def __init__(self, shape, weights, threads: int | None = None):
        """shape: heliopause_b200.model.DecoderShape; weights: SyntheticWeights."""
        self.s = shape
        self.w = weights
        self.threads = threads or o.cpu_threads()
        self._cache = {}
        self.kv = {}

    def _weight(self, layer, slot):
        key = (layer, slot)
        if key not in self._cache:
            t, data = self.w.weight(layer, slot)
            k, r = self.s.weight_shape(slot)
            self._cache[key] = (t, data, o.prepare_scales(t, data, k, r), k, r)
        return self._cache[key]

    def _lm_head(self):
        if "lm" not in self._cache:
            data = self.w.lm_head()
            self._cache["lm"] = (data, o.prepare_scales(o.Q6_K, data, self.s.hidden, self.s.vocab))
        return self._cache["lm"]

    def matmul(self, layer, slot, x, cols):
        t, data, scales, k, r = self._weight(layer, slot)
        return o.matmul_prepared(t, data, scales, x, k, r, cols, threads=self.threads)

    def set_kv(self, kv_layer, kc, vc):
        self.kv[kv_layer] = (np.ascontiguousarray(kc, np.float32), np.ascontiguousarray(vc, np.float32))

    def embed(self, token_ids):
        data, _ = self._lm_head()
        rb = o.row_bytes(o.Q6_K, self.s.hidden)
        rows = [o.dequantize(o.Q6_K, data[t * rb:(t + 1) * rb], self.s.hidden)[0] for t in token_ids]
        return o.scale_embedding(np.concatenate(rows), self.s.hidden)

    def layer(self, l, x, positions):
        s = self.s
        m = len(positions)
        hd, nh, nkv = s.head_dim, s.heads, s.kv_heads
        attn_norm = o.rms_norm_rows(x, self.w.norm(l, 0), s.rms_eps)
        q = self.matmul(l, 0, attn_norm, m)
        qn = o.rms_norm_rows(q, self.w.norm(l, 1), s.rms_eps)
        qr = o.rope_neox(qn, hd, nh, positions, hd, s.rope_theta)
        src = s.kv_source(l)
        if s.has_kv(l):
            kp = self.matmul(l, 1, attn_norm, m)
            vp = self.matmul(l, 2, attn_norm, m)
            kn = o.rms_norm_rows(kp, self.w.norm(l, 2), s.rms_eps)
            vn = o.rms_norm_rows_noweight(vp, hd, s.rms_eps)
            kr = o.rope_neox(kn, hd, nkv, positions, hd, s.rope_theta)
            kc, vc = self.kv[src]
            o.kv_update(kc, vc, s.context, nkv, hd, hd, kr, vn, positions)
        kc, vc = self.kv[src]
        top = max(positions)
        count = min(s.context, top + 1)
        start = top + 1 - count
        # compactKeyCache / compactValueCache (layers.ts:932-965)
        slots = (start + np.arange(count)) % s.context
        kcomp = np.ascontiguousarray(kc[slots])
        vcomp = np.ascontiguousarray(vc[:, :, slots])
        mask = causal_mask(positions, start, count)
        attn = o.gqa_attention(qr, kcomp, vcomp, head=hd, nq=nh, nkv=nkv, ntok=m, nkvtok=count, kvstart=0, cap=count,
                               scale=1.0, value_layout=1, qf16=True, mask=mask)
        attn16 = o.cast_f16_rows(attn)
        op = self.matmul(l, 3, attn16, m)
        # residualAdd (layers.ts:850-859): f32 add of f32 arrays
        h1 = (x + o.rms_norm_rows(op, self.w.norm(l, 3), s.rms_eps)).astype(np.float32)
        ffn_in = o.rms_norm_rows(h1, self.w.norm(l, 4), s.rms_eps)
        gate = self.matmul(l, 4, ffn_in, m)
        up = self.matmul(l, 5, ffn_in, m)
        act = o.geglu(gate, up)
        down = self.matmul(l, 6, act, m)
        return (h1 + o.rms_norm_rows(down, self.w.norm(l, 5), s.rms_eps)).astype(np.float32)

    def forward(self, token_ids, positions, top_k: int):
        """Returns (ids [m][k], values [m][k], final residual [m][hidden])."""
        s = self.s
        m = len(token_ids)
        x = self.embed(token_ids)
        for layer in range(s.layers):
            x = self.layer(layer, x, list(positions))
        norm = o.rms_norm_rows(x, self.w.output_norm(), s.rms_eps)
        data, scales = self._lm_head()
        logits = o.matmul_prepared(o.Q6_K, data, scales, norm, s.hidden, s.vocab, m, threads=self.threads)
        if s.softcap and s.softcap > 0:
            logits = o.softcap(logits, s.softcap)
        ids = np.zeros((m, top_k), np.int32)
        vals = np.zeros((m, top_k), np.float32)
        for i in range(m):
            ids[i], vals[i] = o.topk(logits[i * s.vocab:(i + 1) * s.vocab], top_k)
        return ids, vals, x.reshape(m, s.hidden), logits.reshape(m, s.vocab)
