"""GGUF -> HBM resident loader for the decoder model.

Restates the reference's storage layer for the tensors the CUDA decode path
keeps resident:
  * parseGguf                 packages/engine/src/gguf.ts:149-211
      header (magic "GGUF", version, tensor and metadata counts), the typed
      metadata values (gguf.ts:266-365: u8/i8/u16/i16/u32/i32/f32/bool/
      string/array/u64/i64/f64), tensor infos (name, dims, type, offset) and
      the data section at the next multiple of `general.alignment` (default
      32, gguf.ts:95, 200-205);
  * tensorByteLength          packages/engine/src/tensor-reader.ts:268-280
      (block types: bytes per block x elements / block size);
  * readTensorRangesCoalesced packages/engine/src/tensor-reader.ts:158-266
      tensor ranges sorted by offset and merged when the gap between them is
      small, so a model's many tensors are read in few large reads;
  * buildModelManifest        packages/engine/src/model.ts:340-460
      the gemma4.* keys that shape the decoder (block count, widths, heads,
      shared-KV layers, context, RoPE base, RMS epsilon, final softcap).
The quantized bytes go to the device unchanged; the library repacks them into
its tile layout at upload (hpc_weight_upload).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

MAGIC = b"GGUF"
DEFAULT_ALIGNMENT = 32
COALESCE_GAP = 1 << 20  # merge tensor ranges separated by at most 1 MiB

# ggml type id -> (name, elements per block, bytes per block)
GGML_TYPES = {0: ("F32", 1, 4), 1: ("F16", 1, 2), 8: ("Q8_0", 32, 34), 2: ("Q4_0", 32, 18), 12: ("Q4_K", 256, 144),
              13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210), 23: ("IQ4_XS", 256, 136), 26: ("I32", 1, 4),
              30: ("BF16", 1, 2)}

_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


class GgufError(ValueError):
    pass


@dataclass
class TensorInfo:
    name: str
    dims: list[int]
    type_id: int
    offset: int           # relative to the data section
    data_offset: int = 0  # absolute file offset

    @property
    def type_name(self) -> str:
        return GGML_TYPES.get(self.type_id, (f"UNKNOWN_{self.type_id}",))[0]

    @property
    def n_bytes(self) -> int:
        """tensorByteLength: elements / block size x block bytes."""
        if self.type_id not in GGML_TYPES:
            raise GgufError(f"{self.name}: unsupported ggml type {self.type_id}")
        _, per_block, block_bytes = GGML_TYPES[self.type_id]
        n = 1
        for d in self.dims:
            n *= d
        if n % per_block:
            raise GgufError(f"{self.name}: {n} elements is not a whole number of {per_block}-blocks")
        return n // per_block * block_bytes


@dataclass
class GgufFile:
    path: str
    version: int
    metadata: dict
    tensors: list[TensorInfo]
    data_start: int
    by_name: dict = field(default_factory=dict)

    def tensor(self, name: str) -> TensorInfo:
        if name not in self.by_name:
            raise GgufError(f"tensor {name} not in {self.path}")
        return self.by_name[name]

    def number(self, key: str, default=None):
        v = self.metadata.get(key, default)
        if isinstance(v, list):
            return v
        return v


class _Cursor:
    def __init__(self, f):
        self.f = f
        self.offset = 0

    def read(self, n: int) -> bytes:
        b = self.f.read(n)
        if len(b) != n:
            raise GgufError(f"unexpected end of file at offset {self.offset}")
        self.offset += n
        return b

    def scalar(self, fmt: str):
        return struct.unpack(fmt, self.read(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        n = self.scalar("<Q")
        return self.read(n).decode("utf-8")

    def value(self, type_id: int):
        if type_id in _SCALARS:
            return self.scalar(_SCALARS[type_id])
        if type_id == 8:
            return self.string()
        if type_id == 9:
            elem = self.scalar("<I")
            n = self.scalar("<Q")
            return [self.value(elem) for _ in range(n)]
        raise GgufError(f"unknown metadata value type {type_id} at offset {self.offset}")


def read_gguf(path: str) -> GgufFile:
    """parseGguf (gguf.ts:149-211)."""
    with open(path, "rb") as f:
        c = _Cursor(f)
        magic = c.read(4)
        if magic != MAGIC:
            raise GgufError(f"Invalid GGUF magic: expected GGUF, got {magic!r}")
        version = c.scalar("<I")
        n_tensors = c.scalar("<Q")
        n_meta = c.scalar("<Q")
        metadata = {}
        for _ in range(n_meta):
            key = c.string()
            metadata[key] = c.value(c.scalar("<I"))
        tensors = []
        for _ in range(n_tensors):
            name = c.string()
            nd = c.scalar("<I")
            dims = [c.scalar("<Q") for _ in range(nd)]
            type_id = c.scalar("<I")
            offset = c.scalar("<Q")
            tensors.append(TensorInfo(name, dims, type_id, offset))
        align = int(metadata.get("general.alignment", DEFAULT_ALIGNMENT))
        start = (c.offset + align - 1) // align * align
    for t in tensors:
        t.data_offset = start + t.offset
    g = GgufFile(path, version, metadata, tensors, start)
    g.by_name = {t.name: t for t in tensors}
    return g


def read_tensors_coalesced(g: GgufFile, names, gap: int = COALESCE_GAP) -> dict[str, np.ndarray]:
    """readTensorRangesCoalesced (tensor-reader.ts:158-266): the requested
    tensors' byte ranges sorted by offset, merged while the gap between
    consecutive ranges is <= `gap`, each merged range read once; returns
    name -> uint8 view into the range's buffer."""
    infos = sorted((g.tensor(n) for n in names), key=lambda t: t.data_offset)
    groups: list[list[TensorInfo]] = []
    for t in infos:
        if groups:
            last = groups[-1][-1]
            if t.data_offset - (last.data_offset + last.n_bytes) <= gap:
                groups[-1].append(t)
                continue
        groups.append([t])
    out = {}
    with open(g.path, "rb") as f:
        for grp in groups:
            lo = grp[0].data_offset
            hi = max(t.data_offset + t.n_bytes for t in grp)
            f.seek(lo)
            buf = np.frombuffer(f.read(hi - lo), dtype=np.uint8)
            if buf.size != hi - lo:
                raise GgufError(f"short read of [{lo}, {hi}) in {g.path}")
            for t in grp:
                out[t.name] = buf[t.data_offset - lo:t.data_offset - lo + t.n_bytes]
    return out


def decoder_shape(g: GgufFile):
    """buildModelManifest (model.ts:340-460) for the decoder this path runs:
    every layer full-attention, the last `shared_kv_layers` reusing KV."""
    from .model import DecoderShape
    m = g.metadata
    arch = m.get("general.architecture")
    if arch != "gemma4":
        raise GgufError(f"architecture {arch!r}: the CUDA decode path loads gemma4 decoders")

    def req(key):
        if key not in m:
            raise GgufError(f"Missing GGUF metadata {key}")
        return m[key]
    blocks = int(req("gemma4.block_count"))
    kvh = req("gemma4.attention.head_count_kv")
    kvh = int(kvh[0] if isinstance(kvh, list) else kvh)
    shared = int(m.get("gemma4.attention.shared_kv_layers", 0))
    softcap = m.get("gemma4.final_logit_softcapping")
    return DecoderShape(hidden=int(req("gemma4.embedding_length")), heads=int(req("gemma4.attention.head_count")),
                        kv_heads=kvh, head_dim=int(req("gemma4.attention.key_length")),
                        ffn=int(req("gemma4.feed_forward_length")), vocab=int(g.tensor("token_embd.weight").dims[1]),
                        layers=blocks, kv_layers=blocks - shared, context=int(req("gemma4.context_length")),
                        rms_eps=float(req("gemma4.attention.layer_norm_rms_epsilon")),
                        rope_theta=float(m.get("gemma4.rope.freq_base", 1e6)),
                        softcap=float(softcap) if softcap else 0.0)


def tensor_names(shape) -> list[str]:
    """The resident tensors of the decode path, in model.ts's names."""
    names = ["token_embd.weight", "output_norm.weight"]
    for layer in range(shape.layers):
        p = f"blk.{layer}."
        names += [p + n for n in ("attn_q.weight", "attn_output.weight", "ffn_gate.weight", "ffn_up.weight",
                                  "ffn_down.weight", "attn_norm.weight", "attn_q_norm.weight", "attn_k_norm.weight",
                                  "post_attention_norm.weight", "ffn_norm.weight", "post_ffw_norm.weight")]
        if shape.has_kv(layer):
            names += [p + "attn_k.weight", p + "attn_v.weight"]
    return names


def load_into(model, g: GgufFile) -> None:
    """Uploads every resident tensor of `g` into a CudaDecoderModel built for
    decoder_shape(g): quantized weights through hpc_weight_upload (repacked
    at upload), norms as f32."""
    from .model import N_NAMES, N_OUTPUT, W_NAMES
    s = model.shape
    data = read_tensors_coalesced(g, tensor_names(s))
    type_ids = {12: 1, 14: 3}  # ggml Q4_K / Q6_K -> library type ids
    for layer in range(s.layers):
        for slot in s.slots(layer):
            name = f"blk.{layer}.{W_NAMES[slot]}.weight"
            t = g.tensor(name)
            if t.type_id not in type_ids:
                raise GgufError(f"{name}: {t.type_name} is not resident on this path (Q4_K / Q6_K)")
            k, r = s.weight_shape(slot)
            if t.dims != [k, r]:
                raise GgufError(f"{name}: dims {t.dims}, expected {[k, r]}")
            model.set_weight(layer, slot, type_ids[t.type_id], data[name])
        for slot, n in N_NAMES.items():
            name = f"blk.{layer}.{n}.weight"
            if g.tensor(name).type_id != 0:
                raise GgufError(f"{name} must be F32")
            model.set_norm(layer, slot, data[name].view(np.float32))
    model.set_norm(0, N_OUTPUT, data["output_norm.weight"].view(np.float32))
    emb = g.tensor("token_embd.weight")
    if emb.type_id != 14:
        raise GgufError(f"token_embd.weight: {emb.type_name}; the LM head path is Q6_K")
    model.set_lm_head(data["token_embd.weight"])


def load_model(path: str, max_tokens: int = 8, top_k: int = 64):
    """A CudaDecoderModel resident in HBM from a GGUF file."""
    from .model import CudaDecoderModel
    g = read_gguf(path)
    m = CudaDecoderModel(decoder_shape(g), max_tokens=max_tokens, top_k=top_k)
    try:
        load_into(m, g)
    except Exception:
        m.close()
        raise
    return m
