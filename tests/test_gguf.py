"""GGUF -> HBM loader (heliopause_b200/gguf.py).

The test files are written by gguf-py's GGUFWriter (an implementation
independent of the loader, in the image) from the seeded synthetic weights,
with the gemma4 metadata keys that model.ts reads.

CPU: header, metadata and tensor table round-trip; the decoder shape;
tensor bytes identical to the synthetic source after coalesced reads (and
the reads are coalesced); the reference's error for a bad magic; a
truncated file, an unsupported tensor type, a missing tensor and another
architecture are rejected.

GPU: a model loaded from the file gives bit-identical top-k and hidden
state to the same weights uploaded directly (load_synthetic).
"""
from dataclasses import replace

import numpy as np
import pytest

from heliopause_b200 import gguf as hg
from heliopause_b200.model import N_NAMES, W_NAMES, DecoderShape, SyntheticWeights

SHAPE = DecoderShape(hidden=2048, heads=8, kv_heads=2, head_dim=256, ffn=2048, vocab=4096, layers=3, kv_layers=2,
                     context=64)


def write_gguf(path, shape, weights, *, arch="gemma4", drop=None):
    import gguf
    w = gguf.GGUFWriter(str(path), arch)
    w.add_uint32("gemma4.block_count", shape.layers)
    w.add_uint32("gemma4.embedding_length", shape.hidden)
    w.add_uint32("gemma4.feed_forward_length", shape.ffn)
    w.add_uint32("gemma4.attention.head_count", shape.heads)
    w.add_uint32("gemma4.attention.head_count_kv", shape.kv_heads)
    w.add_uint32("gemma4.attention.key_length", shape.head_dim)
    w.add_uint32("gemma4.attention.value_length", shape.head_dim)
    w.add_uint32("gemma4.context_length", shape.context)
    w.add_uint32("gemma4.attention.shared_kv_layers", shape.layers - shape.kv_layers)
    w.add_float32("gemma4.attention.layer_norm_rms_epsilon", shape.rms_eps)
    w.add_float32("gemma4.rope.freq_base", shape.rope_theta)
    q = {1: gguf.GGMLQuantizationType.Q4_K, 3: gguf.GGMLQuantizationType.Q6_K}
    rb = {1: 144, 3: 210}
    w.add_tensor("token_embd.weight", weights.lm_head().reshape(shape.vocab, -1),
                 raw_dtype=gguf.GGMLQuantizationType.Q6_K)
    w.add_tensor("output_norm.weight", weights.output_norm())
    for layer in range(shape.layers):
        for slot in shape.slots(layer):
            t, data = weights.weight(layer, slot)
            k, r = shape.weight_shape(slot)
            name = f"blk.{layer}.{W_NAMES[slot]}.weight"
            if name == drop:
                continue
            w.add_tensor(name, data.reshape(r, k // 256 * rb[t]), raw_dtype=q[t])
        for slot, n in N_NAMES.items():
            w.add_tensor(f"blk.{layer}.{n}.weight", weights.norm(layer, slot))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.fixture(scope="module")
def gguf_file(tmp_path_factory):
    pytest.importorskip("gguf")
    p = tmp_path_factory.mktemp("gguf") / "tiny.gguf"
    write_gguf(p, SHAPE, SyntheticWeights(SHAPE, seed=3))
    return p


def test_header_metadata_and_shape(gguf_file):
    g = hg.read_gguf(str(gguf_file))
    assert g.version == 3
    assert g.metadata["general.architecture"] == "gemma4"
    assert g.data_start % 32 == 0
    # the file stores the epsilon as f32; the reference reads it as that value
    assert hg.decoder_shape(g) == replace(SHAPE, rms_eps=float(np.float32(SHAPE.rms_eps)))
    assert g.tensor("blk.0.attn_q.weight").dims == [2048, 2048]
    assert g.tensor("blk.0.attn_v.weight").type_name == "Q6_K"  # even layers keep attn_v / ffn_down in Q6_K
    assert g.tensor("blk.1.attn_v.weight").type_name == "Q4_K"
    assert g.tensor("token_embd.weight").dims == [2048, 4096]
    assert "blk.2.attn_k.weight" not in g.by_name  # shared-KV layer


def test_tensor_bytes_round_trip_and_coalescing(gguf_file, monkeypatch):
    g = hg.read_gguf(str(gguf_file))
    w = SyntheticWeights(SHAPE, seed=3)
    reads = []
    real_open = open

    class Spy:
        def __init__(self, f):
            self.f = f

        def __enter__(self):
            return self

        def __exit__(self, *a):
            self.f.close()

        def seek(self, o):
            self.f.seek(o)

        def read(self, n):
            reads.append(n)
            return self.f.read(n)
    monkeypatch.setattr("builtins.open", lambda p, mode="r", *a, **k: Spy(real_open(p, mode, *a, **k)))
    data = hg.read_tensors_coalesced(g, hg.tensor_names(SHAPE))
    monkeypatch.undo()
    assert len(reads) < len(data) // 4, f"{len(reads)} reads for {len(data)} tensors"
    assert np.array_equal(data["token_embd.weight"], w.lm_head())
    assert np.array_equal(data["output_norm.weight"].view(np.float32), w.output_norm())
    for layer in range(SHAPE.layers):
        for slot in SHAPE.slots(layer):
            assert np.array_equal(data[f"blk.{layer}.{W_NAMES[slot]}.weight"], w.weight(layer, slot)[1])
        for slot, n in N_NAMES.items():
            assert np.array_equal(data[f"blk.{layer}.{n}.weight"].view(np.float32), w.norm(layer, slot))


def test_bad_files_are_rejected(gguf_file, tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + gguf_file.read_bytes()[4:64])
    with pytest.raises(hg.GgufError, match="Invalid GGUF magic"):
        hg.read_gguf(str(bad))
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(gguf_file.read_bytes()[:200])
    with pytest.raises(hg.GgufError, match="end of file"):
        hg.read_gguf(str(cut))
    g = hg.read_gguf(str(gguf_file))
    g.tensor("blk.0.attn_q.weight").type_id = 99
    with pytest.raises(hg.GgufError, match="unsupported ggml type"):
        _ = g.tensor("blk.0.attn_q.weight").n_bytes
    with pytest.raises(hg.GgufError, match="not in"):
        g.tensor("blk.9.attn_q.weight")
    missing = tmp_path / "missing.gguf"
    write_gguf(missing, SHAPE, SyntheticWeights(SHAPE, seed=3), drop="blk.1.ffn_up.weight")
    with pytest.raises(hg.GgufError, match="blk.1.ffn_up.weight not in"):
        hg.read_tensors_coalesced(hg.read_gguf(str(missing)), hg.tensor_names(SHAPE))
    other = tmp_path / "llama.gguf"
    write_gguf(other, SHAPE, SyntheticWeights(SHAPE, seed=3), arch="llama")
    with pytest.raises(hg.GgufError, match="architecture"):
        hg.decoder_shape(hg.read_gguf(str(other)))


@pytest.mark.gpu
def test_gguf_model_equals_direct_upload(gguf_file):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from heliopause_b200 import kernels as hk
    from heliopause_b200.model import CudaDecoderModel
    hk.init_device(0)
    w = SyntheticWeights(SHAPE, seed=3)
    a = hg.load_model(str(gguf_file))
    b = CudaDecoderModel(a.shape, max_tokens=8, top_k=64)  # the file's f32 epsilon
    try:
        b.load_synthetic(w)
        for kl in range(SHAPE.kv_layers):
            kc, vc = w.kv(kl, 20)
            for m in (a, b):
                gk, gv = m.kv(kl)
                gk.copy_(torch.from_numpy(kc))
                gv.copy_(torch.from_numpy(vc))
        for toks, pos in (([17], [20]), ([3, 99, 1000, 7, 4000], [21, 22, 23, 24, 25])):
            ia, va, ha = a.forward(toks, pos, 40, return_hidden=True)
            ib, vb, hb = b.forward(toks, pos, 40, return_hidden=True)
            assert torch.equal(ia, ib) and torch.equal(va, vb) and torch.equal(ha, hb)
    finally:
        a.close()
        b.close()
