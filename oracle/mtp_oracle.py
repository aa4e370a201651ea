"""CPU restatement of the MTP draft head and the greedy speculative loop
(parity oracle).

TEST INFRASTRUCTURE ONLY (see oracle.py): imported by tests/ and nowhere in
the product path.

Draft head: packages/engine/src/runner/wasm/mtp-assistant-runner.ts
  runWasmMtpAssistant        :43-66    pre_projection over [embedding ; hidden],
                                       layers, output norm, post_projection,
                                       centroid logits
  forwardAssistantLayer      :68-140   attn norm, q projection + per-head q norm,
                                       partial NeoX RoPE, GQA attention over the
                                       target KV (f32 query, scale 1), o
                                       projection, post-attention norm + residual,
                                       FFN, layer output scale
  forwardAssistantFfn        :142-158  fround(gelu(gate) * up), down, norm, residual
  matMulAssistantWeight      :160-183  f32 matmul of dequantized rows
                                       (lib.rs:103-154 hp_matmul_dequantized_f32)
  maskedEmbeddingTopTokens   :211-242  top centroids -> token ordering -> rows . h
Loop: generateAssistantWithMtp (packages/engine/src/chat.ts:692-776) with
proposeMtpDraft (mtp-generation.ts:92-137), acceptGreedyMtpDraft
(mtp-generation.ts:199-228) and the verify runner's contexts
(webgpu/mtp-target-runner.ts:80-161, normalizedHiddenSlice :225-244).

Parity unpinned: the reference's MTP tests check shapes, plumbing and
determinism of the draft/verify loop, not draft-head values, so this
restatement rests on reading the runner line by line.  The matmuls, attention
and top-k reuse the C restatements pinned in oracle.py.
"""
from __future__ import annotations

import numpy as np

from . import oracle as o


class OracleDraftHead:
    """shape: heliopause_b200.mtp.MtpDraftShape; weights: SyntheticDraftWeights."""

    def __init__(self, shape, weights):
        self.s = shape
        self.w = weights
        self._m = {}

    def _matrix(self, name):
        if name not in self._m:
            t, k, n = self.s.matrices()[name]
            self._m[name] = (t, self.w.matrix(name), k, n)
        return self._m[name]

    def mm(self, name, x) -> np.ndarray:
        t, data, k, n = self._matrix(name)
        return o.matmul_dequantized(t, data, x, k, n, 1)

    def run(self, target_embedding, target_hidden, kv, position: int, top_k: int):
        """Returns (backbone hidden, ids, values).  kv[layer] = (K
        [context][kv_heads][head_dim], V [head_dim][kv_heads][context]) numpy
        arrays of the mapped target layer."""
        s = self.s
        x = self.mm("mtp.pre_projection.weight", np.concatenate([target_embedding, target_hidden]))
        for layer in range(s.layers):
            x = self.layer(layer, x, kv[layer], position)
        h = o.rms_norm_f32sum_rows(x, self.w.vector("output_norm.weight"), s.rms_eps)
        post = self.mm("mtp.post_projection.weight", h)
        cent = self.mm("mtp.centroids.weight", h)
        ids, vals = self.masked_top_tokens(h, cent, top_k)
        return post, ids, vals

    def masked_top_tokens(self, h, centroid_logits, top_k: int):
        """mtp-assistant-runner.ts:211-242."""
        s = self.s
        c_ids, _ = o.topk(centroid_logits, min(s.centroid_top_k, s.n_centroids))
        ordering = self.w.token_ordering()
        per = len(ordering) // s.n_centroids
        seen, sel = set(), []
        for c in c_ids:
            for tok in ordering[c * per:min((c + 1) * per, len(ordering))]:
                tok = int(tok)
                if 0 <= tok < len(ordering) and tok not in seen:
                    seen.add(tok)
                    sel.append(tok)
        t, data, k, n = self._matrix("token_embd.weight")
        rb = o.row_bytes(t, k)
        rows = np.concatenate([data[i * rb:(i + 1) * rb] for i in sel])
        vals = o.matmul_dequantized(t, rows, h, k, len(sel), 1)
        order = sorted(range(len(sel)), key=lambda i: (-float(vals[i]), sel[i]))[:top_k]
        return np.array([sel[i] for i in order], np.int64), np.array([vals[i] for i in order], np.float32)

    def layer(self, layer: int, x, kv, position: int) -> np.ndarray:
        s, w = self.s, self.w
        p = f"blk.{layer}."
        a = o.rms_norm_f32sum_rows(x, w.vector(p + "attn_norm.weight"), s.rms_eps)
        q = o.rms_norm_f32sum_rows(self.mm(p + "attn_q.weight", a), w.vector(p + "attn_q_norm.weight"), s.rms_eps)
        q = o.rope_neox_pairs(q, s.head_dim, s.heads, position, s.head_dim, s.active_pairs, s.rope_theta)
        kc, vc = kv
        count = position + 1
        kcomp = np.ascontiguousarray(kc[:count])
        vcomp = np.ascontiguousarray(vc[:, :, :count])
        att = o.gqa_attention(q, kcomp, vcomp, head=s.head_dim, nq=s.heads, nkv=s.kv_heads, ntok=1, nkvtok=count,
                              kvstart=0, cap=count, scale=1.0, value_layout=1, qf16=False,
                              mask=np.zeros(count, np.float32))
        op = self.mm(p + "attn_output.weight", att)
        r = (x + o.rms_norm_f32sum_rows(op, w.vector(p + "post_attention_norm.weight"), s.rms_eps)).astype(np.float32)
        n = o.rms_norm_f32sum_rows(r, w.vector(p + "ffn_norm.weight"), s.rms_eps)
        act = o.gelu_mul_f32(self.mm(p + "ffn_gate.weight", n), self.mm(p + "ffn_up.weight", n))
        down = self.mm(p + "ffn_down.weight", act)
        f = (r + o.rms_norm_f32sum_rows(down, w.vector(p + "post_ffw_norm.weight"), s.rms_eps)).astype(np.float32)
        return (f.astype(np.float64) * w.layer_output_scale(layer)).astype(np.float32)


def target_embedding(target, token: int) -> np.ndarray:
    """readTargetInputEmbedding (mtp-generation.ts:190-197): the target's
    embedding row * sqrt(D)."""
    return target.embed([token])


def normalized_hidden(target, hidden) -> np.ndarray:
    """normalizedHiddenSlice (webgpu/mtp-target-runner.ts:225-244)."""
    return o.rms_norm_f32sum_rows(hidden, target.w.output_norm(), target.s.rms_eps)


def greedy_proposals(target, draft: OracleDraftHead, kv_layers):
    """proposeMtpDraft with greedy sampling: a callable
    (pending, position, hidden, n) -> draft token ids."""
    def propose(pending, position, hidden, n):
        drafts, tok, h = [], pending, hidden
        kv = [target.kv[kl] for kl in kv_layers]
        for _ in range(n):
            post, ids, _ = draft.run(target_embedding(target, tok), h, kv, position, 1)
            tok = int(ids[0])
            drafts.append(tok)
            h = post
        return drafts
    return propose


def greedy_mtp_generate(target, propose, first_token: int, ctx_position: int, ctx_hidden, n_tokens: int,
                        n_spec: int):
    """Greedy generateAssistantWithMtp on the oracle decoder (target:
    oracle.decoder_oracle.OracleDecoder); `propose` as greedy_proposals
    returns.  Returns (tokens, rounds, accepted drafts)."""
    out, rounds, accepted = [], 0, 0
    pending, pos = first_token, ctx_position + 1
    position, hidden = ctx_position, ctx_hidden
    while len(out) < n_tokens and pos < target.s.context:
        budget = max(0, min(n_spec, n_tokens - len(out) - 1, target.s.context - pos - 1))
        drafts = list(propose(pending, position, hidden, budget)) if budget else []
        tokens = [pending] + drafts
        ids, _, x, _ = target.forward(tokens, [pos + i for i in range(len(tokens))], 1)
        tops = [int(r[0]) for r in ids]
        n_acc = 0
        while n_acc < len(drafts) and drafts[n_acc] == tops[n_acc]:
            n_acc += 1
        committed = 1 + n_acc
        rounds += 1
        accepted += n_acc
        out.extend(tokens[:committed][:n_tokens - len(out)])
        position = pos + committed - 1
        hidden = normalized_hidden(target, x[committed - 1])
        pos += committed
        pending = tops[n_acc]
    return out, rounds, accepted
