"""MTP speculative decoding on the GPU: the draft head ("MTP assistant") and
the draft / batched-verify / accept loop.

The draft head restates runWasmMtpAssistant
(packages/engine/src/runner/wasm/mtp-assistant-runner.ts:43-242; the WebGPU
runner, runner/webgpu/mtp-assistant-runner.ts, computes the same in f32):

    x      = pre_projection @ [target embedding ; target current hidden]
    per layer (attention over the TARGET's KV cache, model.ts:457-478 layer map):
      a    = rmsNorm(x, attn_norm);  q = normHeads(Wq a, q_norm);  q = RoPE(q)
             (full-attention NeoX, only floor(nDims * 0.25 / 2) pairs rotated)
      o    = Wo gqa_attention(q, K, V, causal, scale 1)
      r    = x + rmsNorm(o, post_attention_norm)
      f    = r + rmsNorm(Wd fround(gelu(Wg n) * (Wu n)), post_ffw_norm),  n = rmsNorm(r, ffn_norm)
      x    = fround(f * layer_output_scale)
    h      = rmsNorm(x, output_norm)
    backbone hidden = post_projection @ h
    top tokens = maskedEmbeddingTopTokens(h, centroids @ h): the top
             centroid_top_k centroids select token ids through token_ordering,
             scored by their embedding rows . h (value desc, id asc).

The step runs in the library (hpc_draft_step, csrc/hc_draft.cu: one CUDA
graph of its own kernels).  All matmuls are f32 products of dequantized
weights with f32 inputs, as hp_matmul_dequantized_f32 (lib.rs:103-154) / the
WebGPU F32 matmul do: every weight element is dequantized bit-exactly from
the head's resident quantized tiles and each output row is one sequential
f32 chain in index order.  The norms, RoPE, attention softmax (f64 exp, f32
query) and GELU follow the reference's rounding points; the norm and
attention sums run in parallel orders, so those agree to f32 rounding.

The loop (mtp_generate) restates generateAssistantWithMtp
(packages/engine/src/chat.ts:692-776) with proposeMtpDraft
(mtp-generation.ts:92-137): drafts from the pending token at the context's
constant position, one batched verify of [pending, d1..dn] through
CudaDecoderModel.forward, acceptance by generation.accept_mtp_draft, and the
next context from the verify's hidden at the last committed position
(finalizeMtpVerification; normalizedHiddenSlice,
webgpu/mtp-target-runner.ts:225-244).  By default each draft is drawn on the
device (hpc_sample_candidates, the host sampler's steps and generator
stream) and the verify reads the drafts where the sampler wrote them, so a
round synchronizes with the host once, after the verify.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from . import generation as gen
from . import kernels as hk
from . import synthetic as syn


@dataclass(frozen=True)
class MtpDraftShape:
    backbone: int = 2048        # target hidden size
    hidden: int = 2048          # draft head width
    heads: int = 8
    kv_heads: int = 2           # equals the target's KV heads
    head_dim: int = 256
    ffn: int = 8192
    vocab: int = 262144
    n_centroids: int = 2048
    centroid_top_k: int = 32
    layers: int = 1
    rope_theta: float = 1.0e6
    rms_eps: float = 1e-6

    @property
    def active_pairs(self) -> int:
        """Rotated pairs of a full-attention layer (mtp-assistant-runner.ts:96)."""
        return int(math.floor(self.head_dim * 0.25 / 2))

    def matrices(self):
        """name -> (type, K, N) of every quantized matrix (token_embd: rows = vocab)."""
        E, D, Hq = self.hidden, self.backbone, self.heads * self.head_dim
        m = {"mtp.pre_projection.weight": (syn.Q4_K, 2 * D, E), "mtp.post_projection.weight": (syn.Q4_K, E, D),
             "mtp.centroids.weight": (syn.Q4_K, E, self.n_centroids), "token_embd.weight": (syn.Q6_K, E, self.vocab)}
        for layer in range(self.layers):
            m[f"blk.{layer}.attn_q.weight"] = (syn.Q4_K, E, Hq)
            m[f"blk.{layer}.attn_output.weight"] = (syn.Q4_K, Hq, E)
            m[f"blk.{layer}.ffn_gate.weight"] = (syn.Q4_K, E, self.ffn)
            m[f"blk.{layer}.ffn_up.weight"] = (syn.Q4_K, E, self.ffn)
            m[f"blk.{layer}.ffn_down.weight"] = (syn.Q4_K, self.ffn, E)
        return m

    def vectors(self):
        """name -> length of every f32 norm vector."""
        v = {"output_norm.weight": self.hidden}
        for layer in range(self.layers):
            for n in ("attn_norm", "post_attention_norm", "ffn_norm", "post_ffw_norm"):
                v[f"blk.{layer}.{n}.weight"] = self.hidden
            v[f"blk.{layer}.attn_q_norm.weight"] = self.head_dim
        return v


class SyntheticDraftWeights:
    """Seeded draft head (BASELINE distributions): quantized fields uniform,
    norms 1 + N(0, 0.1), layer output scale 1 + N(0, 0.1), token ordering a
    seeded permutation of the vocabulary."""

    def __init__(self, shape: MtpDraftShape, seed: int = 7):
        self.s, self.seed = shape, seed

    def matrix(self, name: str) -> np.ndarray:
        t, k, n = self.s.matrices()[name]
        return syn.quant_weight(t, n, k, seed=self.seed * 1000 + sum(map(ord, name)))

    def vector(self, name: str) -> np.ndarray:
        g = syn.rng(self.seed * 7919 + sum(map(ord, name)))
        return (1.0 + 0.1 * g.standard_normal(self.s.vectors()[name])).astype(np.float32)

    def layer_output_scale(self, layer: int) -> float:
        g = syn.rng(self.seed * 31 + layer)
        return float(np.float32(1.0 + 0.1 * g.standard_normal()))

    def token_ordering(self) -> np.ndarray:
        return syn.rng(self.seed * 13).permutation(self.s.vocab).astype(np.int32)


def target_kv_layer(target_layers: int, target_kv_layers: int, draft_layers: int, draft_layer: int) -> int:
    """mapMtpAssistantLayerToTargetKvLayer (model.ts:457-478) for a target
    whose layers are all full-attention and whose first target_kv_layers own
    a KV cache."""
    bucket = min(target_layers - 1, (draft_layer + 1) * target_layers // draft_layers - 1)
    for layer in range(bucket, -1, -1):
        if layer < target_kv_layers:
            return layer
    raise ValueError(f"no target KV layer at or before depth {bucket}")


# ---- f32 arithmetic with the reference's rounding points -------------------

def _rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """rmsNorm over the last dimension (mtp-assistant-runner.ts:275-290): f32
    sum of squares, f64 scale, fround(fround(x * scale) * w)."""
    ss = torch.sum(x * x, dim=-1, keepdim=True)  # f32
    scale = 1.0 / torch.sqrt(ss.double() / x.shape[-1] + eps)
    return ((x.double() * scale).float().double() * w.double()).float()


# draft matrix / vector names -> library ids (include/heliocuda.h HPC_DW_* / HPC_DN_*)
_DW = {"mtp.pre_projection.weight": 100, "mtp.post_projection.weight": 101, "mtp.centroids.weight": 102,
       "token_embd.weight": 103, "attn_q.weight": 0, "attn_output.weight": 1, "ffn_gate.weight": 2,
       "ffn_up.weight": 3, "ffn_down.weight": 4}
_DN = {"output_norm.weight": 100, "attn_norm.weight": 0, "attn_q_norm.weight": 1, "post_attention_norm.weight": 2,
       "ffn_norm.weight": 3, "post_ffw_norm.weight": 4}
DRAFT_CONTEXT = 4096  # positions the draft head accepts (the target's context may be smaller)


def _split_name(name: str) -> tuple[int, str]:
    """'blk.{layer}.{rest}' -> (layer, rest); head-wide names -> (0, name)."""
    if name.startswith("blk."):
        _, layer, rest = name.split(".", 2)
        return int(layer), rest
    return 0, name


class CudaMtpDraftHead:
    """The draft head resident on the current CUDA device (hpc_draft_*): each
    matrix kept as quantized row tiles and multiplied with
    hp_matmul_dequantized_f32's arithmetic (bit-exact dequantization, one
    sequential f32 chain per row), one step per CUDA graph."""

    def __init__(self, shape: MtpDraftShape, weights: SyntheticDraftWeights, *, gpu_seed: int | None = None,
                 max_top_k: int = 64):
        """gpu_seed: generate the quantized matrices on the device (same
        distributions, for benchmark-size heads) instead of weights.matrix."""
        import ctypes as C

        from . import _lib
        self.s = shape
        self._C, self._L = C, _lib.lib()
        self.max_top_k = max_top_k
        cfg = _lib.DraftConfig(shape.backbone, shape.hidden, shape.heads, shape.kv_heads, shape.head_dim, shape.ffn,
                               shape.vocab, shape.n_centroids, shape.centroid_top_k, shape.layers, DRAFT_CONTEXT,
                               max_top_k, shape.rms_eps, shape.rope_theta)
        h = C.c_void_p()
        hk.assert_cuda_ok(self._L.hpc_draft_create(C.byref(cfg), C.byref(h)), "draftCreate")
        self._h = h
        try:
            gen_ = None
            if gpu_seed is not None:
                from .model import gpu_synthetic_weight
                gen_ = torch.Generator(device="cuda")
                gen_.manual_seed(gpu_seed)
            for name, (t, k, n) in shape.matrices().items():
                data = weights.matrix(name) if gen_ is None else gpu_synthetic_weight(t, n, k, gen_)
                wh = hk.create_quantized_weight_handle("Q4_K" if t == syn.Q4_K else "Q6_K", data, k, n)
                try:
                    layer, rest = _split_name(name)
                    hk.assert_cuda_ok(self._L.hpc_draft_set_matrix(self._h, _DW[rest], layer, wh.handle),
                                      f"draftSetMatrix {name}")
                finally:
                    hk.release_quantized_weight_handle(wh)
            for name in shape.vectors():
                v = np.ascontiguousarray(weights.vector(name), np.float32)
                layer, rest = _split_name(name)
                hk.assert_cuda_ok(self._L.hpc_draft_set_vector(self._h, _DN[rest], layer, v.ctypes.data, v.size),
                                  f"draftSetVector {name}")
            for layer in range(shape.layers):
                hk.assert_cuda_ok(self._L.hpc_draft_set_layer_scale(self._h, layer,
                                                                    C.c_float(weights.layer_output_scale(layer))),
                                  "draftSetLayerScale")
            order = np.ascontiguousarray(weights.token_ordering(), np.int32)
            hk.assert_cuda_ok(self._L.hpc_draft_set_token_ordering(self._h, order.ctypes.data, order.size),
                              "draftSetTokenOrdering")
        except Exception:
            self.close()
            raise
        self._kv_keep = []
        self.post = torch.empty(shape.backbone, device="cuda")
        self.ids = torch.empty(max_top_k, dtype=torch.int32, device="cuda")
        self.vals = torch.empty(max_top_k, device="cuda")

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._L.hpc_draft_release(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def run(self, target_embedding: torch.Tensor, target_hidden: torch.Tensor, kv, position: int, top_k: int):
        """One draft step: (backbone hidden [backbone], ids, logits [top_k]),
        on the device.  kv[layer] = (K [context][kv_heads][head_dim], V in the
        reference orientation [head_dim][kv_heads][context]) of the mapped
        target layer; V is used token-major (a view of the model's own
        storage when it is one, else a contiguous copy)."""
        C = self._C
        keep = []
        for layer, (k, v) in enumerate(kv):
            k = k.contiguous()
            vt = v.permute(2, 1, 0)
            if not vt.is_contiguous():
                vt = vt.contiguous()
            keep += [k, vt]
            hk.assert_cuda_ok(self._L.hpc_draft_set_target_kv(self._h, layer, C.c_void_p(k.data_ptr()),
                                                              C.c_void_p(vt.data_ptr())), "draftSetTargetKv")
        self._kv_keep = keep
        emb = target_embedding.to(device="cuda", dtype=torch.float32).contiguous()
        hid = target_hidden.to(device="cuda", dtype=torch.float32).contiguous()
        st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        hk.assert_cuda_ok(self._L.hpc_draft_step(self._h, C.c_void_p(emb.data_ptr()), C.c_void_p(hid.data_ptr()),
                                                 int(position), int(top_k), C.c_void_p(self.post.data_ptr()),
                                                 C.c_void_p(self.ids.data_ptr()), C.c_void_p(self.vals.data_ptr()),
                                                 st), "draftStep")
        return self.post.clone(), self.ids[:top_k].long(), self.vals[:top_k].clone()


# ---- the speculative decoding loop ------------------------------------------

@dataclass
class MtpContext:
    position: int
    current_hidden: torch.Tensor  # normalized target hidden (f32 [backbone])


def normalized_hidden(hidden: torch.Tensor, output_norm: torch.Tensor, eps: float) -> torch.Tensor:
    """normalizedHiddenSlice (webgpu/mtp-target-runner.ts:225-244)."""
    return _rms_norm(hidden, output_norm, eps)


class MtpGenerator:
    """Target model + draft head + embedding table for the draft inputs."""

    def __init__(self, target, draft: CudaMtpDraftHead):
        """target: a loaded CudaDecoderModel (its tied embedding / LM head and
        output norm feed the draft head's inputs)."""
        self.t, self.d, self.ts = target, draft, target.shape
        ds, ts = draft.s, target.shape
        # validateMtpAssistantCompatibility (mtp-generation.ts:60-90) and the
        # KV head size check of validateTargetKvLayer (mtp-assistant-runner.ts:258-273)
        if ds.backbone != ts.hidden:
            raise ValueError(f"MTP assistant backbone hidden size {ds.backbone} does not match target hidden size "
                             f"{ts.hidden}.")
        if ds.kv_heads != ts.kv_heads:
            raise ValueError(f"MTP assistant KV head count {ds.kv_heads} does not match target KV head count "
                             f"{ts.kv_heads}.")
        if ds.vocab != ts.vocab:
            raise ValueError(f"MTP assistant vocabulary size {ds.vocab} does not match target vocabulary size "
                             f"{ts.vocab}.")
        if ds.head_dim != ts.head_dim:
            raise ValueError(f"Target KV head size mismatch for assistant layer 0: {ts.head_dim}/{ts.head_dim}")
        self.embd = hk.dequantize_resident(target.lm_head_handle)  # [vocab][hidden] f32
        self.out_norm = torch.from_numpy(target.output_norm_values).cuda()
        ts = self.ts
        self.kv_layers = [target_kv_layer(ts.layers, ts.kv_layers, draft.s.layers, i) for i in range(draft.s.layers)]

    def embedding(self, token: int) -> torch.Tensor:
        """readTargetInputEmbedding (mtp-generation.ts:190-197): row * sqrt(D), f32."""
        return (self.embd[token].double() * math.sqrt(self.ts.hidden)).float()

    def context_at(self, position: int, hidden: torch.Tensor) -> MtpContext:
        """MtpTargetContext of a target position from its final residual."""
        return MtpContext(position, normalized_hidden(hidden, self.out_norm, self.ts.rms_eps))

    def start(self, token: int, position: int, sampling, rng):
        """The prefill's last step (MtpTargetPrefillResult): forward `token`
        at `position`, sample the first pending token from its top-k
        distribution (chat.ts:700) and return it with the context there."""
        ids, vals, hid = self.t.forward([token], [position], self.target_top_k(sampling), return_hidden=True)
        dist = gen.MtpTokenDistribution(list(zip(ids[0].tolist(), vals[0].tolist())), self.ts.vocab)
        return gen.sample_mtp_token_distribution(dist, sampling, rng), self.context_at(position, hid[0])

    @staticmethod
    def target_top_k(sampling) -> int:
        """Candidates the verify forward reads back per position
        (sampling.logitsTopK, chat.ts:730)."""
        return sampling.logits_top_k or (1 if gen._greedy(sampling) else max(1, sampling.top_k))

    def propose(self, pending: int, ctx: MtpContext, n: int, sampling, rng):
        """proposeMtpDraft (mtp-generation.ts:92-137): constant position and
        target KV, the backbone hidden fed back."""
        kv = [self.t.kv(layer) for layer in self.kv_layers]
        drafts, dists = [], []
        token, hidden = pending, ctx.current_hidden
        k = 1 if gen._greedy(sampling) else sampling.top_k  # mtpDraftTopK (mtp-generation.ts:230-234)
        for _ in range(n):
            post, ids, logits = self.d.run(self.embedding(token), hidden, kv, ctx.position, k)
            pairs = list(zip(ids.tolist(), logits.tolist()))
            token = gen.sample_next_token([gen.Candidate(i, v) for i, v in pairs], sampling, rng)
            drafts.append(token)
            dists.append(gen.MtpTokenDistribution(pairs, self.d.s.vocab, True))
            hidden = post
        return gen.MtpProposal(drafts, dists)

    def propose_on_device(self, pending: int, ctx: MtpContext, n: int, sampling, rng):
        """proposeMtpDraft with every draw on the device (hpc_sample_candidates):
        each draft step's top-k, its token and the next step's input
        embedding stay on the GPU, so the n steps run without a host
        synchronization.  Returns the device tokens [n] (int32) and the
        steps' (ids, logits) device tensors; the host stream `rng` is
        advanced past the n draws."""
        kv = [self.t.kv(layer) for layer in self.kv_layers]
        greedy = gen._greedy(sampling)
        k = 1 if greedy else sampling.top_k  # mtpDraftTopK (mtp-generation.ts:230-234)
        toks = torch.empty(n, dtype=torch.int32, device="cuda")
        emb, hidden = self.embedding(pending), ctx.current_hidden
        scale = math.sqrt(self.ts.hidden)
        steps = []
        for i in range(n):
            post, ids, logits = self.d.run(emb, hidden, kv, ctx.position, k)
            ids32 = ids.to(torch.int32)
            nxt = torch.empty(self.ts.hidden, dtype=torch.float32, device="cuda")
            hk.sample_candidates(ids32, logits, top_k=k if greedy else sampling.top_k, top_p=sampling.top_p,
                                 temperature=sampling.temperature if not greedy else 1.0, greedy=greedy,
                                 rng_state=0 if greedy else rng.state(), token_out=toks[i:i + 1], table=self.embd,
                                 scale=scale, row_out=nxt)
            if not greedy:
                rng()  # this copy of the stream moves past the device's draw
            steps.append((ids32, logits))
            emb, hidden = nxt, post
        return toks, steps

    def verify(self, tokens, position: int, top_k: int):
        """verifyMtpDraft: one batched target forward over [pending, d1..dn]
        at positions position.. (webgpu/mtp-target-runner.ts:80-149)."""
        ids, vals, hid = self.t.forward(tokens, [position + i for i in range(len(tokens))], top_k, return_hidden=True)
        return gen.target_verification(ids.cpu().numpy(), vals.cpu().numpy(), self.ts.vocab, position), hid

    def verify_device(self, pending: int, toks: torch.Tensor, steps, position: int, top_k: int):
        """verify() on device draft tokens: the forward reads them where the
        sampler wrote them; the one read-back of the round brings the
        target's top-k, the drafts and their distributions together."""
        n = toks.numel()
        ids_dev = torch.cat([torch.full((1,), pending, dtype=torch.int32, device="cuda"), toks])
        pos_dev = torch.arange(position, position + n + 1, dtype=torch.int32, device="cuda")
        ids, vals, hid = self.t.forward_device(ids_dev, pos_dev, top_k, return_hidden=True)
        d_ids = torch.stack([s[0] for s in steps]).cpu().tolist()
        d_vals = torch.stack([s[1] for s in steps]).cpu().tolist()
        drafts = toks.cpu().tolist()
        prop = gen.MtpProposal(drafts, [gen.MtpTokenDistribution(list(zip(i, v)), self.d.s.vocab, True)
                                        for i, v in zip(d_ids, d_vals)])
        return gen.target_verification(ids.cpu().numpy(), vals.cpu().numpy(), self.ts.vocab, position), hid, prop

    def generate(self, first_token: int, ctx: MtpContext, n_tokens: int, n_spec: int, sampling, rng, *,
                 device_sampling: bool = True):
        """generateAssistantWithMtp (chat.ts:692-776) without tokenizer and
        stop tokens: `first_token` is the pending token at ctx.position + 1.
        Returns (tokens, rounds, accepted drafts).  device_sampling: the
        drafts are drawn on the GPU and fed straight into the verify forward,
        one host synchronization per round (after the verify); else the host
        draws each draft (one synchronization per draft)."""
        out, rounds, accepted = [], 0, 0
        pending, pos = first_token, ctx.position + 1
        top_k = self.target_top_k(sampling)
        while len(out) < n_tokens and pos < self.ts.context:
            budget = max(0, min(n_spec, n_tokens - len(out) - 1, self.ts.context - pos - 1))
            if device_sampling and budget:
                toks, steps = self.propose_on_device(pending, ctx, budget, sampling, rng)
                ver, hid, prop = self.verify_device(pending, toks, steps, pos, top_k)
            else:
                prop = self.propose(pending, ctx, budget, sampling, rng) if budget else gen.MtpProposal([], [])
                ver, hid = self.verify([pending] + prop.draft_token_ids, pos, top_k)
            acc = gen.accept_mtp_draft(prop, ver, sampling, rng)
            rounds += 1
            accepted += acc.accepted_draft_length
            committed = [pending] + prop.draft_token_ids[:acc.accepted_draft_length]
            out.extend(committed[:n_tokens - len(out)])
            ctx = self.context_at(pos + acc.committed_length - 1, hid[acc.committed_length - 1])
            pos += acc.committed_length
            pending = acc.next_token_id
        return out, rounds, accepted
