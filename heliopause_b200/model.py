"""Resident decoder model on the GPU: the CUDA counterpart of the reference's
model runner for the decode hot path.

Reference interfaces mirrored here (paths inside the Heliopause tree):
  * ModelRunner.decodeToken / SegmentRunner.runTokenHidden
    (packages/engine/src/runner/model-runner.ts:54-73,
     runner/segment-runner.ts:18-34): `CudaDecoderModel.decode_token`
  * MtpTargetRunner.verify (runner/mtp-target-runner.ts:59-82, WebGPU
    implementation runner/webgpu/mtp-target-runner.ts:80-149): one batched
    forward over [pending, ...drafts] with per-position top-k:
    `CudaDecoderModel.forward` with token_count = 1 + drafts
  * forwardOutput (runner/wasm/layers.ts:381-416): the top-k of every call.

The model shape is Gemma-4-like (35 layers, hidden 2048,
8 query / 2 KV heads of 256, FFN 16384 GEGLU, the last 15 layers reuse the KV
of layer 19, Q4_K weights with Q6_K attn_v / ffn_down on even layers, tied
Q6_K embedding / LM head of 262,144 rows, fp32 KV cache).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, replace

import numpy as np
import torch

from . import _lib
from . import kernels as hk
from . import synthetic as syn

W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN = range(7)
N_ATTN, N_Q, N_K, N_POST_ATTN, N_FFN, N_POST_FFW = range(6)
N_OUTPUT = 100
W_NAMES = {W_Q: "attn_q", W_K: "attn_k", W_V: "attn_v", W_O: "attn_output", W_GATE: "ffn_gate", W_UP: "ffn_up",
           W_DOWN: "ffn_down"}
N_NAMES = {N_ATTN: "attn_norm", N_Q: "attn_q_norm", N_K: "attn_k_norm", N_POST_ATTN: "post_attention_norm",
           N_FFN: "ffn_norm", N_POST_FFW: "post_ffw_norm"}


@dataclass(frozen=True)
class DecoderShape:
    hidden: int = 2048
    heads: int = 8
    kv_heads: int = 2
    head_dim: int = 256
    ffn: int = 16384
    vocab: int = 262144
    layers: int = 35
    kv_layers: int = 20
    context: int = 4096
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    softcap: float = 0.0

    def weight_shape(self, slot: int) -> tuple[int, int]:
        """(input_size K, row_count N) of a weight slot."""
        qd = self.heads * self.head_dim
        kvd = self.kv_heads * self.head_dim
        return {W_Q: (self.hidden, qd), W_K: (self.hidden, kvd), W_V: (self.hidden, kvd), W_O: (qd, self.hidden),
                W_GATE: (self.hidden, self.ffn), W_UP: (self.hidden, self.ffn), W_DOWN: (self.ffn, self.hidden)}[slot]

    def weight_type(self, layer: int, slot: int) -> int:
        """Q4_K_M mix: attn_v and ffn_down are Q6_K on even layers."""
        if slot in (W_V, W_DOWN) and layer % 2 == 0:
            return syn.Q6_K
        return syn.Q4_K

    def has_kv(self, layer: int) -> bool:
        return layer < self.kv_layers

    def kv_source(self, layer: int) -> int:
        """kvSourceLayers (engine/src/model.ts:382-388), all layers full-attention."""
        return layer if layer < self.kv_layers else self.kv_layers - 1

    def slots(self, layer: int):
        return [s for s in range(7) if self.has_kv(layer) or s not in (W_K, W_V)]

    def weight_bytes(self) -> int:
        n = syn.row_bytes(syn.Q6_K, self.hidden) * self.vocab
        for layer in range(self.layers):
            for s in self.slots(layer):
                k, r = self.weight_shape(s)
                n += syn.row_bytes(self.weight_type(layer, s), k) * r
        return n

    def kv_read_bytes(self, position: int) -> int:
        """Bytes of K and V one token's attention reads at `position`, all layers."""
        count = min(self.context, position + 1)
        return self.layers * 2 * count * self.kv_heads * self.head_dim * 4


CONFIG3 = DecoderShape()


def _seed(layer: int, slot: int, base: int) -> int:
    return base * 1_000_003 + layer * 101 + slot + 7


class SyntheticWeights:
    """Deterministic GGUF-format weights for a DecoderShape (numpy PCG64)."""

    def __init__(self, shape: DecoderShape, seed: int = 1):
        self.shape = shape
        self.seed = seed

    def weight(self, layer: int, slot: int) -> tuple[int, np.ndarray]:
        k, r = self.shape.weight_shape(slot)
        t = self.shape.weight_type(layer, slot)
        return t, syn.quant_weight(t, r, k, _seed(layer, slot, self.seed))

    def lm_head(self) -> np.ndarray:
        return syn.q6_k_weight(self.shape.vocab, self.shape.hidden, _seed(999, 0, self.seed))

    def norm(self, layer: int, slot: int) -> np.ndarray:
        """RMSNorm weights ~ 1 + N(0, 0.1)."""
        n = self.shape.head_dim if slot in (N_Q, N_K) else self.shape.hidden
        g = syn.rng(_seed(layer, 50 + slot, self.seed))
        return (1.0 + 0.1 * g.standard_normal(n)).astype(np.float32)

    def output_norm(self) -> np.ndarray:
        g = syn.rng(_seed(998, 0, self.seed))
        return (1.0 + 0.1 * g.standard_normal(self.shape.hidden)).astype(np.float32)

    def kv(self, kv_layer: int, filled: int) -> tuple[np.ndarray, np.ndarray]:
        """fp32 KV ~ N(0,1) for positions [0, filled); zeros elsewhere.
        K [context][kv_heads][head_dim], V [head_dim][kv_heads][context]."""
        s = self.shape
        g = syn.rng(_seed(kv_layer, 90, self.seed))
        kc = np.zeros((s.context, s.kv_heads, s.head_dim), np.float32)
        vc = np.zeros((s.head_dim, s.kv_heads, s.context), np.float32)
        kc[:filled] = g.standard_normal((filled, s.kv_heads, s.head_dim), dtype=np.float32)
        vc[:, :, :filled] = g.standard_normal((s.head_dim, s.kv_heads, filled), dtype=np.float32)
        return kc, vc


def gpu_synthetic_weight(type_id: int, rows: int, k: int, gen: torch.Generator) -> torch.Tensor:
    """Same distributions as synthetic.quant_weight, generated on the GPU (for
    benchmark-size models; not bit-identical to the numpy generator)."""
    nb = rows * (k // 256)
    if type_id == syn.Q4_K:
        blk = torch.randint(0, 256, (nb, 144), dtype=torch.uint8, device="cuda", generator=gen)
        d = (torch.randn(nb, device="cuda", generator=gen).abs() * 0.01).half().view(torch.uint8).view(nb, 2)
        dm = (torch.randn(nb, device="cuda", generator=gen).abs() * 0.005).half().view(torch.uint8).view(nb, 2)
        blk[:, 0:2] = d
        blk[:, 2:4] = dm
        # 12 scale bytes from uniform 6-bit scales/mins: random bytes already are
        # a valid packing of uniform 6-bit values (every bit pattern decodes).
        return blk.reshape(-1)
    blk = torch.randint(0, 256, (nb, 210), dtype=torch.uint8, device="cuda", generator=gen)
    blk[:, 208:210] = (torch.randn(nb, device="cuda", generator=gen).abs() * 0.01).half().view(torch.uint8).view(nb, 2)
    return blk.reshape(-1)


class CudaDecoderModel:
    """A DecoderShape resident in HBM behind hpc_model_* (include/heliocuda.h)."""

    def __init__(self, shape: DecoderShape, max_tokens: int = 8, top_k: int = 64):
        self.shape = shape
        self.max_tokens = max_tokens
        self.top_k = top_k
        cfg = _lib.ModelConfig(shape.hidden, shape.heads, shape.kv_heads, shape.head_dim, shape.ffn, shape.vocab,
                               shape.layers, shape.kv_layers, shape.context, max_tokens, top_k, shape.rms_eps,
                               shape.rope_theta, shape.softcap)
        h = C.c_void_p()
        hk.assert_cuda_ok(_lib.lib().hpc_model_create(C.byref(cfg), C.byref(h)), "modelCreate")
        self._h = h
        self.handles: list[hk.CudaQuantizedWeightHandle] = []
        self.weight_handles: dict[tuple[int, int], hk.CudaQuantizedWeightHandle] = {}
        self._ids = torch.empty(max_tokens, dtype=torch.int32, device="cuda")
        self._pos = torch.empty(max_tokens, dtype=torch.int32, device="cuda")
        self.out_ids = torch.empty((max_tokens, top_k), dtype=torch.int32, device="cuda")
        self.out_vals = torch.empty((max_tokens, top_k), dtype=torch.float32, device="cuda")
        self.hidden = torch.empty((max_tokens, shape.hidden), dtype=torch.float32, device="cuda")

    # ---- loading -----------------------------------------------------------
    def set_weight(self, layer: int, slot: int, type_id: int, data) -> None:
        k, r = self.shape.weight_shape(slot)
        name = "Q6_K" if type_id == syn.Q6_K else "Q4_K"
        h = hk.create_quantized_weight_handle(name, data, k, r)
        self.handles.append(h)
        self.weight_handles[(layer, slot)] = h
        hk.assert_cuda_ok(_lib.lib().hpc_model_set_weight(self._h, layer, slot, h.handle), "modelSetWeight")

    def set_norm(self, layer: int, slot: int, values: np.ndarray) -> None:
        v = np.ascontiguousarray(values, np.float32)
        if slot == N_OUTPUT:
            self.output_norm_values = v.copy()
        hk.assert_cuda_ok(_lib.lib().hpc_model_set_norm(self._h, layer, slot, v.ctypes.data_as(C.c_void_p), v.size),
                          "modelSetNorm")

    def set_lm_head(self, data) -> None:
        h = hk.create_quantized_weight_handle("Q6_K", data, self.shape.hidden, self.shape.vocab)
        self.handles.append(h)
        self.lm_head_handle = h
        hk.assert_cuda_ok(_lib.lib().hpc_model_set_lm_head(self._h, h.handle), "modelSetLmHead")

    def load_synthetic(self, weights: SyntheticWeights) -> None:
        s = self.shape
        for layer in range(s.layers):
            for slot in s.slots(layer):
                t, data = weights.weight(layer, slot)
                self.set_weight(layer, slot, t, data)
            for slot in range(6):
                self.set_norm(layer, slot, weights.norm(layer, slot))
        self.set_norm(0, N_OUTPUT, weights.output_norm())
        self.set_lm_head(weights.lm_head())

    def load_gpu_synthetic(self, seed: int = 1) -> None:
        """Benchmark-size model generated on the GPU (same distributions)."""
        s = self.shape
        gen = torch.Generator(device="cuda")
        gen.manual_seed(seed)
        w = SyntheticWeights(s, seed)
        for layer in range(s.layers):
            for slot in s.slots(layer):
                k, r = s.weight_shape(slot)
                t = s.weight_type(layer, slot)
                self.set_weight(layer, slot, t, gpu_synthetic_weight(t, r, k, gen))
            for slot in range(6):
                self.set_norm(layer, slot, w.norm(layer, slot))
        self.set_norm(0, N_OUTPUT, w.output_norm())
        self.set_lm_head(gpu_synthetic_weight(syn.Q6_K, s.vocab, s.hidden, gen))

    def fill_kv_random(self, filled: int, seed: int = 3) -> None:
        """KV ~ N(0,1) for positions [0, filled) of every KV layer (on the GPU)."""
        gen = torch.Generator(device="cuda")
        gen.manual_seed(seed)
        for kl in range(self.shape.kv_layers):
            k, v = self.kv(kl)
            k.zero_()
            v.zero_()
            k[:filled].normal_(generator=gen)
            v[:, :, :filled].normal_(generator=gen)

    def kv(self, kv_layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Views of one KV layer's cache in the reference's orientation: K
        [context][kv_heads][head_dim] and V [head_dim][kv_heads][context]
        (layers.ts:887-911).  The device stores V token-major
        ([context][kv_heads][head_dim], like K), so the V view is a permuted,
        non-contiguous view of that storage."""
        k = C.c_void_p()
        v = C.c_void_p()
        hk.assert_cuda_ok(_lib.lib().hpc_model_kv(self._h, kv_layer, C.byref(k), C.byref(v)), "modelKv")
        s = self.shape
        n = s.context * s.kv_heads * s.head_dim
        kt = _wrap_device(k.value, n).view(s.context, s.kv_heads, s.head_dim)
        vt = _wrap_device(v.value, n).view(s.context, s.kv_heads, s.head_dim).permute(2, 1, 0)
        return kt, vt

    # ---- running -----------------------------------------------------------
    def set_exact(self, enable: bool) -> None:
        """Reference-order steps (default; bit-identical top-k) or the
        reordered kernels (hpc_model_set_exact)."""
        hk.assert_cuda_ok(_lib.lib().hpc_model_set_exact(self._h, int(bool(enable))), "modelSetExact")

    def forward(self, token_ids, positions, top_k: int, *, return_hidden: bool = False):
        """Top-k (ids, values) of every position, [n][top_k] torch tensors."""
        ids = torch.as_tensor(token_ids, dtype=torch.int32).reshape(-1)
        pos = torch.as_tensor(positions, dtype=torch.int32).reshape(-1)
        n = ids.numel()
        if n != pos.numel() or not 1 <= n <= self.max_tokens:
            raise hk.CudaKernelError(hk.ERR_SHAPE, f"forward: {n} tokens / {pos.numel()} positions")
        self._ids[:n].copy_(ids, non_blocking=True)
        self._pos[:n].copy_(pos, non_blocking=True)
        st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        code = _lib.lib().hpc_model_forward(self._h, C.c_void_p(self._ids.data_ptr()), C.c_void_p(self._pos.data_ptr()),
                                            n, top_k, C.c_void_p(self.out_ids.data_ptr()),
                                            C.c_void_p(self.out_vals.data_ptr()),
                                            C.c_void_p(self.hidden.data_ptr()) if return_hidden else None, st)
        hk.assert_cuda_ok(code, "modelForward")
        # the library writes [n][top_k] contiguously; return copies so later
        # calls do not overwrite what the caller holds
        ids_out = self.out_ids.view(-1)[:n * top_k].view(n, top_k).clone()
        vals_out = self.out_vals.view(-1)[:n * top_k].view(n, top_k).clone()
        if return_hidden:
            return ids_out, vals_out, self.hidden[:n].clone()
        return ids_out, vals_out

    def forward_device(self, ids: torch.Tensor, positions: torch.Tensor, top_k: int, *,
                       return_hidden: bool = False):
        """forward() on device int32 token ids and positions (no host copy in
        either direction): what a device-side sampler feeds the verify."""
        n = ids.numel()
        if n != positions.numel() or not 1 <= n <= self.max_tokens:
            raise hk.CudaKernelError(hk.ERR_SHAPE, f"forward: {n} tokens / {positions.numel()} positions")
        self._ids[:n].copy_(ids.reshape(-1).to(torch.int32), non_blocking=True)
        self._pos[:n].copy_(positions.reshape(-1).to(torch.int32), non_blocking=True)
        st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        code = _lib.lib().hpc_model_forward(self._h, C.c_void_p(self._ids.data_ptr()), C.c_void_p(self._pos.data_ptr()),
                                            n, top_k, C.c_void_p(self.out_ids.data_ptr()),
                                            C.c_void_p(self.out_vals.data_ptr()),
                                            C.c_void_p(self.hidden.data_ptr()) if return_hidden else None, st)
        hk.assert_cuda_ok(code, "modelForward")
        ids_out = self.out_ids.view(-1)[:n * top_k].view(n, top_k).clone()
        vals_out = self.out_vals.view(-1)[:n * top_k].view(n, top_k).clone()
        if return_hidden:
            return ids_out, vals_out, self.hidden[:n].clone()
        return ids_out, vals_out

    def prefill(self, hidden: torch.Tensor, start: int) -> torch.Tensor:
        """SegmentRunner.runTokensHidden for a prompt: `hidden` [n][hidden]
        (f32, the embedded tokens) at positions start .. start+n-1 through all
        layers (hpc_model_prefill).  Writes the tokens' K/V and returns the
        final residual stream [n][hidden]."""
        x = hidden.to(device="cuda", dtype=torch.float32).contiguous().reshape(-1, self.shape.hidden)
        n = x.shape[0]
        pos = torch.arange(start, start + n, dtype=torch.int32, device="cuda")
        out = torch.empty_like(x)
        st = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        hk.assert_cuda_ok(_lib.lib().hpc_model_prefill(self._h, C.c_void_p(x.data_ptr()), C.c_void_p(pos.data_ptr()),
                                                       n, C.c_void_p(out.data_ptr()), st), "modelPrefill")
        return out

    def decode_token(self, token_id: int, position: int, top_k: int):
        """ModelRunner.decodeToken: one token -> its top-k candidates."""
        ids, vals = self.forward([token_id], [position], top_k)
        return ids[0], vals[0]

    def close(self) -> None:
        if self._h:
            _lib.lib().hpc_model_release(self._h)
            self._h = None
        for h in self.handles:
            hk.release_quantized_weight_handle(h)
        self.handles.clear()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _wrap_device(ptr: int, n: int) -> torch.Tensor:
    """A float32 CUDA tensor aliasing n floats at a device pointer the model owns."""
    class _Holder:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}
    return torch.as_tensor(_Holder(), device="cuda")
