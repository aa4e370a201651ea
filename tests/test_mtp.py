"""MTP draft head and the draft / batched-verify / accept loop.

CPU (oracle/mtp_oracle.py, the C restatement of the draft-head math):
  * mapMtpAssistantLayerToTargetKvLayer (model.ts:457-478) for the config-3
    target, the partial-RoPE pair count (mtp-assistant-runner.ts:96);
  * the draft-head helpers against float64 evaluations of their formulas;
  * the draft head is deterministic (the reference's own smoke test,
    test/mtp-assistant.test.ts:82-92) and its masked top tokens equal a
    brute-force numpy selection;
  * greedy speculative decoding emits exactly the target's greedy tokens
    whatever the drafts are -- with the draft head, with drafts that are all
    right and with drafts wrong at planted indices.

GPU (heliopause_b200/mtp.py through the library's dequantization and the
decoder C-ABI):
  * one draft step equals the oracle's: backbone hidden within
    |gpu - ref| <= 1e-3 (|ref| + rms(ref)), top tokens identical except near-ties;
  * MtpGenerator greedy tokens equal plain greedy decoding on the same model
    (draft head drafts, all-right drafts, planted wrong drafts), and the
    oracle's speculative loop where no step is a near-tie;
  * sampled generation (temperature 1, seeded uniforms) is deterministic;
  * the device sampler draws the host sampler's token (300 candidate lists),
    and generation with the drafts drawn on the device equals generation
    with the host drawing them.
"""
import math

import numpy as np
import pytest
import torch

from heliopause_b200 import generation as gen
from heliopause_b200.model import CONFIG3, CudaDecoderModel, DecoderShape, SyntheticWeights
from heliopause_b200.mtp import MtpDraftShape, SyntheticDraftWeights, target_kv_layer

TINY_T = DecoderShape(hidden=256, heads=2, kv_heads=1, head_dim=256, ffn=512, vocab=512, layers=2, kv_layers=1,
                      context=48)
TINY_D = MtpDraftShape(backbone=256, hidden=256, heads=2, kv_heads=1, head_dim=256, ffn=256, vocab=512,
                       n_centroids=16, centroid_top_k=4)


def test_target_kv_layer_mapping():
    assert target_kv_layer(CONFIG3.layers, CONFIG3.kv_layers, 1, 0) == 19
    assert [target_kv_layer(35, 20, 4, i) for i in range(4)] == [7, 16, 19, 19]
    assert [target_kv_layer(4, 4, 2, i) for i in range(2)] == [1, 3]
    with pytest.raises(ValueError):
        target_kv_layer(4, 0, 1, 0)


def test_active_pairs():
    assert MtpDraftShape().active_pairs == 32       # floor(256 * 0.25 / 2)
    assert TINY_D.active_pairs == 32


def test_draft_math_helpers(oracle):
    o = oracle
    g = np.random.default_rng(1)
    # rope: position 0 is the identity; only the first `pairs` pairs move
    x = g.standard_normal(2 * 16).astype(np.float32)
    assert np.array_equal(o.rope_neox_pairs(x, 16, 2, 0, 16, 2, 1e4), x)
    r = o.rope_neox_pairs(x, 16, 2, 5, 16, 2, 1e4)
    for h in range(2):
        row, rr = x[h * 16:(h + 1) * 16], r[h * 16:(h + 1) * 16]
        moved = [0, 1, 8, 9]
        assert np.array_equal(np.delete(rr, moved), np.delete(row, moved))
        th = [5.0, float(np.float32(5.0 * 1e4 ** (-2 / 16)))]
        for i in range(2):
            want0 = row[i] * math.cos(th[i]) - row[8 + i] * math.sin(th[i])
            want1 = row[i] * math.sin(th[i]) + row[8 + i] * math.cos(th[i])
            assert abs(rr[i] - want0) <= 1e-6 * (1 + abs(want0))
            assert abs(rr[8 + i] - want1) <= 1e-6 * (1 + abs(want1))
    # gelu: |x| >= 10 short-circuits, otherwise the tanh form
    v = np.array([-12, -10, -3, -0.5, 0, 0.25, 1, 4, 10, 12], np.float32)
    got = o.gelu_mul_f32(v, np.full(v.size, 2, np.float32))
    for xi, gi in zip(v.astype(np.float64), got):
        want = 0.0 if xi <= -10 else xi if xi >= 10 else \
            0.5 * xi * (1 + math.tanh(math.sqrt(2 / math.pi) * (xi + 0.044715 * xi ** 3)))
        assert abs(gi - 2 * want) <= 2e-6 * (1 + abs(want))
    # rms norm with the f32 sum of squares
    x = g.standard_normal((3, 64)).astype(np.float32)
    w = (1 + 0.1 * g.standard_normal(64)).astype(np.float32)
    got = o.rms_norm_f32sum_rows(x, w, 1e-6).reshape(3, 64)
    want = x / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6) * w
    assert np.allclose(got, want, rtol=1e-5, atol=1e-6)


def _tiny_kv(filled, seed=4):
    g = np.random.default_rng(seed)
    k = np.zeros((TINY_T.context, 1, 256), np.float32)
    v = np.zeros((256, 1, TINY_T.context), np.float32)
    k[:filled] = g.standard_normal((filled, 1, 256))
    v[:, :, :filled] = g.standard_normal((256, 1, filled))
    return k, v


def test_oracle_draft_head_deterministic_and_masked_selection(oracle):
    from oracle.mtp_oracle import OracleDraftHead
    w = SyntheticDraftWeights(TINY_D, seed=3)
    d = OracleDraftHead(TINY_D, w)
    g = np.random.default_rng(2)
    emb = g.standard_normal(256).astype(np.float32)
    hid = g.standard_normal(256).astype(np.float32)
    kv = [_tiny_kv(20)]
    a = d.run(emb, hid, kv, 19, 8)
    b = d.run(emb, hid, kv, 19, 8)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1]) and np.array_equal(a[2], b[2])
    assert a[0].shape == (256,) and len(a[1]) == 8
    # masked selection against a brute-force restatement
    h = g.standard_normal(256).astype(np.float32)
    cent = g.standard_normal(TINY_D.n_centroids).astype(np.float32)
    ids, vals = d.masked_top_tokens(h, cent, 10)
    top_c = np.argsort(-cent.astype(np.float64), kind="stable")[:TINY_D.centroid_top_k]
    per = TINY_D.vocab // TINY_D.n_centroids
    order = w.token_ordering()
    toks = sorted({int(t) for c in top_c for t in order[c * per:(c + 1) * per]})
    t, data, k, _ = d._matrix("token_embd.weight")
    table = oracle.dequantize(t, data, k, TINY_D.vocab).reshape(TINY_D.vocab, k).astype(np.float64)
    scores = table[toks] @ h.astype(np.float64)
    want = [toks[i] for i in np.argsort(-scores, kind="stable")[:10]]
    assert list(ids) == want
    assert np.allclose(vals, np.sort(scores)[::-1][:10], rtol=1e-4, atol=1e-4)


def _oracle_target(seed=7, filled=12):
    from oracle.decoder_oracle import OracleDecoder
    w = SyntheticWeights(TINY_T, seed)
    ref = OracleDecoder(TINY_T, w, threads=1)
    for kl in range(TINY_T.kv_layers):
        kc, vc = w.kv(kl, filled)
        ref.set_kv(kl, kc.copy(), vc.copy())
    return ref


def _oracle_greedy(ref, token, position, n):
    """Plain greedy decoding: the tokens at position+1 .. position+n."""
    out = []
    for i in range(n):
        ids, _, _, _ = ref.forward([token], [position + i], 1)
        token = int(ids[0, 0])
        out.append(token)
    return out


def test_oracle_greedy_mtp_equals_greedy_decoding(oracle):
    from oracle import mtp_oracle as mo
    n, start = 14, 11
    plain = _oracle_greedy(_oracle_target(), 5, start, n + 1)
    seq = {start + 1 + i: t for i, t in enumerate(plain)}  # position -> greedy token there

    def run(make_propose):
        ref = _oracle_target()
        ids, _, x, _ = ref.forward([5], [start], 1)
        ctx_h = mo.normalized_hidden(ref, x[0])
        return mo.greedy_mtp_generate(ref, make_propose(ref), int(ids[0, 0]), start, ctx_h, n, 4)

    # drafts from the draft head (random weights: nearly all rejected)
    head = mo.OracleDraftHead(TINY_D, SyntheticDraftWeights(TINY_D, seed=3))
    toks, rounds, acc = run(lambda ref: mo.greedy_proposals(ref, head, [0]))
    assert toks == plain[:n]

    # all-right drafts: every round commits budget + 1 tokens
    def right(pending, position, hidden, k):
        return [seq[position + 2 + i] for i in range(k)]
    toks, rounds, acc = run(lambda ref: right)
    assert toks == plain[:n] and rounds == math.ceil(n / 5) and acc == n - rounds

    # drafts wrong at planted indices: acceptance stops there, output unchanged
    calls = []

    def planted(pending, position, hidden, k):
        d = right(pending, position, hidden, k)
        bad = len(calls) % max(1, k)
        calls.append(bad)
        if d:
            d[bad] = (d[bad] + 1) % TINY_T.vocab
        return d
    toks, rounds, acc = run(lambda ref: planted)
    assert toks == plain[:n] and acc == sum(calls)


# ------------------------------------------------------------------- GPU ----

SMALL_T = DecoderShape(hidden=2048, heads=8, kv_heads=2, head_dim=256, ffn=2048, vocab=4096, layers=3, kv_layers=2,
                       context=64)
SMALL_D = MtpDraftShape(backbone=2048, hidden=1024, heads=4, kv_heads=2, head_dim=256, ffn=2048, vocab=4096,
                        n_centroids=64, centroid_top_k=8)


@pytest.fixture(scope="module")
def gpu_device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from heliopause_b200 import kernels as hk
    hk.init_device(0)


def _gpu_target(seed=3, filled=20):
    w = SyntheticWeights(SMALL_T, seed)
    m = CudaDecoderModel(SMALL_T, max_tokens=8, top_k=64)
    m.load_synthetic(w)
    for kl in range(SMALL_T.kv_layers):
        kc, vc = w.kv(kl, filled)
        gk, gv = m.kv(kl)
        gk.copy_(torch.from_numpy(kc))
        gv.copy_(torch.from_numpy(vc))
    torch.cuda.synchronize()
    return m, w


@pytest.mark.gpu
def test_draft_step_matches_oracle(gpu_device):
    from heliopause_b200.mtp import CudaMtpDraftHead
    from oracle.mtp_oracle import OracleDraftHead
    dw = SyntheticDraftWeights(SMALL_D, seed=5)
    head = CudaMtpDraftHead(SMALL_D, dw)
    ref = OracleDraftHead(SMALL_D, dw)
    g = np.random.default_rng(9)
    kc = g.standard_normal((SMALL_T.context, 2, 256)).astype(np.float32)
    vc = g.standard_normal((256, 2, SMALL_T.context)).astype(np.float32)
    kv_gpu = [(torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda())]
    for trial, position in enumerate([0, 17, 63]):
        emb = g.standard_normal(2048).astype(np.float32)
        hid = g.standard_normal(2048).astype(np.float32)
        post_g, ids_g, vals_g = head.run(torch.from_numpy(emb).cuda(), torch.from_numpy(hid).cuda(), kv_gpu,
                                         position, 16)
        post_r, ids_r, vals_r = ref.run(emb, hid, [(kc, vc)], position, 16)
        post_g = post_g.cpu().numpy()
        scale = np.sqrt(np.mean(post_r.astype(np.float64) ** 2))
        assert np.all(np.abs(post_g - post_r) <= 1e-3 * (np.abs(post_r) + scale)), f"trial {trial}"
        ids_g, vals_g = ids_g.cpu().numpy(), vals_g.cpu().numpy()
        tol = 1e-3 * (np.abs(vals_r) + 1)
        assert np.all(np.abs(vals_g - vals_r) <= tol), f"trial {trial}: values"
        for i in range(16):
            if ids_g[i] != ids_r[i]:  # only a near-tie may reorder
                assert abs(vals_r[i] - vals_g[i]) <= tol[i] and \
                    (i + 1 < 16 and abs(vals_r[i] - vals_r[i + 1]) <= 2 * tol[i] or
                     i > 0 and abs(vals_r[i] - vals_r[i - 1]) <= 2 * tol[i]), f"trial {trial}: id {i}"


def _gpu_plain_greedy(m, token, position, n):
    out = []
    for i in range(n):
        ids, _ = m.decode_token(token, position + i, 1)
        token = int(ids[0])
        out.append(token)
    return out


@pytest.mark.gpu
def test_mtp_greedy_equals_plain_greedy(gpu_device):
    from heliopause_b200.mtp import CudaMtpDraftHead, MtpGenerator
    n, start = 24, 19
    a, _ = _gpu_target()
    try:
        plain = _gpu_plain_greedy(a, 42, start, n + 1)
    finally:
        a.close()
    seq = {start + 1 + i: t for i, t in enumerate(plain)}
    greedy = gen.resolve_generation_sampling_options(do_sample=False)
    head = CudaMtpDraftHead(SMALL_D, SyntheticDraftWeights(SMALL_D, seed=5))

    class Planted(MtpGenerator):
        wrong_at = None

        def propose(self, pending, ctx, k, sampling, rng):
            d = [seq[ctx.position + 2 + i] for i in range(k)]
            if self.wrong_at is not None and d:
                j = self.wrong_at % k
                d[j] = (d[j] + 1) % SMALL_T.vocab
                self.wrong_at += 1
            return gen.MtpProposal(d, [])

    for kind in ("draft head", "all right", "planted"):
        m, _ = _gpu_target()
        try:
            g = (MtpGenerator if kind == "draft head" else Planted)(m, head)
            if kind == "planted":
                g.wrong_at = 0
            first, ctx = g.start(42, start, greedy, gen.create_deterministic_rng(1))
            assert first == plain[0]
            # the planted proposals replace the host-side proposer
            toks, rounds, acc = g.generate(first, ctx, n, 4, greedy, gen.create_deterministic_rng(1),
                                           device_sampling=kind == "draft head")
            assert toks == plain[:n], f"{kind}: {toks} vs {plain[:n]}"
            if kind == "all right":
                assert rounds == math.ceil(n / 5) and acc == n - rounds
            print(kind, "rounds", rounds, "accepted", acc)
        finally:
            m.close()


@pytest.mark.gpu
def test_mtp_generator_validates_compatibility(gpu_device):
    from dataclasses import replace

    from heliopause_b200.mtp import CudaMtpDraftHead, MtpGenerator
    m, _ = _gpu_target()
    try:
        for bad, msg in ((dict(vocab=8192), "vocabulary size"), (dict(kv_heads=1, heads=2), "KV head count"),
                         (dict(backbone=1024), "backbone hidden size")):
            shape = replace(SMALL_D, **bad)
            head = CudaMtpDraftHead.__new__(CudaMtpDraftHead)
            head.s = shape
            with pytest.raises(ValueError, match=msg):
                MtpGenerator(m, head)
    finally:
        m.close()


@pytest.mark.gpu
def test_mtp_sampled_generation_is_deterministic(gpu_device):
    from heliopause_b200.mtp import CudaMtpDraftHead, MtpGenerator
    head = CudaMtpDraftHead(SMALL_D, SyntheticDraftWeights(SMALL_D, seed=5))
    opt = gen.resolve_generation_sampling_options(do_sample=True, temperature=1.0, top_k=40, top_p=1.0, seed=1234)
    runs = []
    for _ in range(2):
        m, _ = _gpu_target()
        try:
            g = MtpGenerator(m, head)
            rng = gen.create_deterministic_rng(opt.seed)
            first, ctx = g.start(42, 19, opt, rng)
            runs.append(g.generate(first, ctx, 20, 4, opt, rng))
        finally:
            m.close()
    assert runs[0] == runs[1]
    toks, rounds, acc = runs[0]
    assert len(toks) == 20 and 1 <= rounds <= 20 and 0 <= acc <= 20 - rounds


@pytest.mark.gpu
def test_device_sampler_equals_host_sampler(gpu_device):
    """hpc_sample_candidates against sample_next_token (generation.ts:85-165)
    on the same candidate lists and generator state: the same token, over
    list lengths 1..200, ties (id ascending), top-k / top-p / temperature and
    greedy; the row written for the next step is table[token] * scale."""
    from heliopause_b200 import kernels as hk
    g = np.random.default_rng(3)
    table = torch.from_numpy(g.standard_normal((5000, 64)).astype(np.float32)).cuda()
    tok = torch.empty(1, dtype=torch.int32, device="cuda")
    row = torch.empty(64, dtype=torch.float32, device="cuda")
    for trial in range(300):
        n = int(g.choice([1, 2, 5, 40, 64, 200]))
        vals = g.normal(0, float(g.choice([0.5, 2.0, 8.0])), n).astype(np.float32)
        if trial % 7 == 0 and n > 3:
            vals[1:3] = vals[0]
        ids = g.permutation(5000)[:n].astype(np.int32)
        order = sorted(range(n), key=lambda i: (-float(vals[i]), int(ids[i])))
        vals, ids = vals[order].copy(), ids[order].copy()
        top_k = int(g.choice([1, 5, 40, 64, 1000]))
        top_p = float(g.choice([0.5, 0.9, 0.95, 1.0]))
        temp = float(g.choice([0.3, 1.0, 1.7]))
        greedy = trial % 11 == 0
        opt = gen.resolve_generation_sampling_options(do_sample=not greedy, temperature=temp, top_p=top_p,
                                                      top_k=top_k, seed=trial)
        rng = gen.create_deterministic_rng(int(g.integers(0, 2 ** 32)))
        for _ in range(trial % 3):
            rng()
        state = rng.state()
        host = gen.sample_next_token([gen.Candidate(int(i), float(v)) for i, v in zip(ids, vals)], opt, rng)
        hk.sample_candidates(torch.from_numpy(ids).cuda(), torch.from_numpy(vals).cuda(), top_k=opt.top_k,
                             top_p=top_p, temperature=temp, greedy=greedy, rng_state=state, token_out=tok,
                             table=table, scale=math.sqrt(64), row_out=row)
        assert int(tok.item()) == host, f"trial {trial}"
        want = (table[host].double() * math.sqrt(64)).float()
        assert torch.equal(row, want), f"trial {trial}: row"
    # a token outside the table leaves the row as it was
    small = table[:100].contiguous()
    row.fill_(7.0)
    hk.sample_candidates(torch.tensor([4321], dtype=torch.int32, device="cuda"),
                         torch.tensor([1.0], dtype=torch.float32, device="cuda"), top_k=1, top_p=1.0,
                         temperature=1.0, greedy=True, rng_state=0, token_out=tok, table=small, scale=1.0, row_out=row)
    assert int(tok.item()) == 4321 and bool(torch.all(row == 7.0))


@pytest.mark.gpu
def test_mtp_device_sampling_equals_host_sampling(gpu_device):
    """The drafts drawn on the device (one synchronization per round) give
    the same generation as the host drawing each draft: same tokens, rounds
    and accepted drafts from the same seed."""
    from heliopause_b200.mtp import CudaMtpDraftHead, MtpGenerator
    head = CudaMtpDraftHead(SMALL_D, SyntheticDraftWeights(SMALL_D, seed=5))
    opt = gen.resolve_generation_sampling_options(do_sample=True, temperature=1.0, top_k=40, top_p=0.95, seed=99)
    runs = []
    for device in (False, True):
        m, _ = _gpu_target()
        try:
            g = MtpGenerator(m, head)
            rng = gen.create_deterministic_rng(opt.seed)
            first, ctx = g.start(42, 19, opt, rng)
            runs.append(g.generate(first, ctx, 24, 4, opt, rng, device_sampling=device))
        finally:
            m.close()
    assert runs[0] == runs[1]


@pytest.mark.gpu
def test_draft_head_rejects_bad_use(gpu_device):
    """hpc_draft_* validation through the C-ABI: a shape it cannot run, a step
    before the weights and target KV are set, a matrix of the wrong shape,
    and top-k / position outside the configured range each return their
    status code (nothing is launched)."""
    import ctypes as C

    from heliopause_b200 import _lib
    from heliopause_b200 import kernels as hk
    L = _lib.lib()
    s = TINY_D
    cfg = _lib.DraftConfig(s.backbone, s.hidden, s.heads, s.kv_heads, s.head_dim, s.ffn, s.vocab, s.n_centroids,
                           s.centroid_top_k, s.layers, 64, 16, s.rms_eps, s.rope_theta)
    bad = _lib.DraftConfig.from_buffer_copy(cfg)
    bad.head_dim = 128
    h = C.c_void_p()
    assert L.hpc_draft_create(C.byref(bad), C.byref(h)) == hk.ERR_SHAPE
    assert L.hpc_draft_create(C.byref(cfg), C.byref(h)) == hk.OK
    try:
        x = torch.zeros(s.backbone, device="cuda")
        post = torch.empty(s.backbone, device="cuda")
        ids = torch.empty(16, dtype=torch.int32, device="cuda")
        vals = torch.empty(16, device="cuda")

        def step(position, k):
            return L.hpc_draft_step(h, C.c_void_p(x.data_ptr()), C.c_void_p(x.data_ptr()), position, k,
                                    C.c_void_p(post.data_ptr()), C.c_void_p(ids.data_ptr()),
                                    C.c_void_p(vals.data_ptr()), None)
        assert step(3, 4) == hk.ERR_ARG  # weights not loaded
        w = SyntheticDraftWeights(s, seed=3)
        t, k, n = s.matrices()["mtp.post_projection.weight"]
        wrong = hk.create_quantized_weight_handle("Q4_K", w.matrix("mtp.post_projection.weight"), k, n)
        try:  # the post projection given as the pre projection (K = 2 * backbone expected)
            assert L.hpc_draft_set_matrix(h, 100, 0, wrong.handle) == hk.ERR_SHAPE
        finally:
            hk.release_quantized_weight_handle(wrong)
        assert step(64, 4) == hk.ERR_SHAPE   # position past the context
        assert step(3, 0) == hk.ERR_SHAPE    # top-k 0
        assert step(3, 17) == hk.ERR_SHAPE   # top-k above max_top_k
    finally:
        assert L.hpc_draft_release(h) == hk.OK
