"""Benchmark for the Heliopause decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Prints ONE JSON line (rank 0).  For N > 1 launch under torchrun; each rank
runs its own replica/shard and the reported time is the max over ranks.

Workloads (a "step" is one pass of the hot path over one batch of synthetic
input, inputs resident in HBM when the timed region starts):
  decode-config3 (default) one decode token of the BASELINE config-3 model
                 (35 layers, hidden 2048, Q4_K_M mix, fp32 KV at context 4096,
                 Q6_K LM head 2048 -> 262,144 with top-40): 3.357 GB of weights
                 and KV per token, far above the 126 MB L2, so every step
                 streams from HBM.  Also reports the M=5 batched verify.
  gemv-config1   one Q4_K GEMV, K=2048 -> N=16384, M=1;
                 rotates 8 weight copies (151 MB > 126 MB L2) so every step
                 streams its weights from HBM.

--impl reference times the reference's CPU implementation of the same step:
the C restatement of the WASM kernels (oracle/, the reference itself cannot
run here), row-sharded over all host threads like the WASM thread pool.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tok/s (E4B-shape Q4_K_M, M=1 & verify M=5); Q4_K GEMV HBM GB/s vs peak"
L2_BYTES = 126 * 1024 * 1024


def _peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.skip = 0
        self.t = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # nvidia-smi takes a moment to start: wait (up to 5 s) for its
            # first sample so that the timed region is covered
            t0 = time.perf_counter()
            while not self.lines and time.perf_counter() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.01)
            self.skip = len(self.lines)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.t:
            self.t.join(timeout=2)

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines[self.skip:] or self.lines[-1:]:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------- workloads ---

class GemvConfig1:
    """Q4_K K=2048 -> N=16384, M=1."""
    name = "gemv-config1"
    K, N, M = 2048, 16384, 1
    copies = 8
    launches_per_step = 2  # Q8_K quantize + GEMV

    def __init__(self):
        import torch

        from heliopause_b200 import kernels as hk
        from heliopause_b200 import synthetic as syn
        self.torch, self.hk, self.syn = torch, hk, syn
        self.w_bytes = syn.row_bytes(syn.Q4_K, self.K) * self.N
        self.algo_bytes = self.w_bytes + 4 * self.K * self.M + 4 * self.N * self.M
        self.handles = [hk.create_quantized_weight_handle("Q4_K", syn.q4_k_weight(self.N, self.K, seed=1000 + i),
                                                          self.K, self.N) for i in range(self.copies)]
        self.x = torch.from_numpy(syn.activations(self.M, self.K, seed=7)).cuda()
        self.out = torch.empty(self.N * self.M, device="cuda")
        import ctypes as C
        from heliopause_b200 import _lib
        self.C, self.L = C, _lib.lib()
        nbytes = C.c_size_t()
        self.L.hpc_q8_workspace_bytes(self.K, self.M, C.byref(nbytes))
        self.ws_bytes = nbytes.value
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device="cuda")
        self.i = 0

    def step(self, ev=None):
        C, L, hk = self.C, self.L, self.hk
        st = C.c_void_p(self.torch.cuda.current_stream().cuda_stream)
        h = self.handles[self.i % self.copies]
        self.i += 1
        hk.assert_cuda_ok(L.hpc_q8_quantize(C.c_void_p(self.x.data_ptr()), self.x.numel(), self.K, self.M,
                                            C.c_void_p(self.ws.data_ptr()), self.ws_bytes, st), "q8")
        hs = (C.c_void_p * 1)(h.handle)
        outs = (C.c_void_p * 1)(self.out.data_ptr())
        lens = (C.c_size_t * 1)(self.out.numel())
        if ev is not None:
            ev[0].record()
        hk.assert_cuda_ok(L.hpc_matmul_q8(1, hs, C.c_void_p(self.ws.data_ptr()), self.ws_bytes, self.K, self.M,
                                          outs, lens, st), "gemv")
        if ev is not None:
            ev[1].record()

    def e2e_step(self, host_x):
        """Public API with host buffers: H2D input, GEMV, D2H output."""
        h = self.handles[self.i % self.copies]
        self.i += 1
        self.hk.mat_mul_quantized_resident(h, host_x, self.K, self.N, self.M)

    def units_per_step(self) -> float:
        return self.algo_bytes / 1e9  # GB per step

    def kernel_launch_count(self) -> int:
        return self.launches_per_step

    def roofline(self, peak_gbs: float) -> dict:
        C, L, hk, torch = self.C, self.L, self.hk, self.torch
        launches = []
        for h in self.handles:
            def f(h=h):
                hs = (C.c_void_p * 1)(h.handle)
                outs = (C.c_void_p * 1)(self.out.data_ptr())
                lens = (C.c_size_t * 1)(self.out.numel())
                hk.assert_cuda_ok(L.hpc_matmul_q8(1, hs, C.c_void_p(self.ws.data_ptr()), self.ws_bytes, self.K,
                                                  self.M, outs, lens,
                                                  C.c_void_p(torch.cuda.current_stream().cuda_stream)), "gemv")
            launches.append(f)
        ms = graph_launch_times(launches * 2)
        achieved = self.algo_bytes / (ms / 1e3) / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s", "frac": achieved / peak_gbs,
                "traffic": None, "kernel": "hc_gemvw_kernel<1> (Q4_K 2048 -> 16384, M=1, reference f32 order)",
                "algorithmic_bytes_per_launch": self.algo_bytes, "launch_ms": ms}

    unit = "GB/s"
    dtype = "u8"

    def config(self) -> dict:
        return {"workload": "Q4_K GEMV K=2048 N=16384 M=1 (BASELINE config 1)", "K": self.K, "N": self.N,
                "M": self.M, "weight_copies_rotated": self.copies,
                "l2": f"inputs larger than L2: {self.copies} weight copies = "
                      f"{self.copies * self.w_bytes / 1e6:.0f} MB rotated per step"}

    def cpu_baseline(self, budget_s: float, threads: int) -> dict:
        from oracle import oracle
        w = self.syn.q4_k_weight(self.N, self.K, seed=1000)
        s = oracle.prepare_scales(oracle.Q4_K, w, self.K, self.N)
        x = self.syn.activations(self.M, self.K, seed=7)
        oracle.matmul_prepared(oracle.Q4_K, w, s, x, self.K, self.N, self.M, threads=threads)  # warm
        n, t0 = 0, time.perf_counter()
        while True:
            oracle.matmul_prepared(oracle.Q4_K, w, s, x, self.K, self.N, self.M, threads=threads)
            n += 1
            dt = time.perf_counter() - t0
            if dt >= budget_s or n >= 2000:
                break
        return {"value": self.algo_bytes * n / dt / 1e9, "unit": self.unit, "cores": threads,
                "kind": "port", "sample": f"{n} config-1 GEMVs in {dt:.1f} s (C restatement of lib.rs, "
                                          f"rows split over {threads} threads like the WASM pool)"}


def graph_launch_times(launches, reps: int = 5) -> float:
    """Average device time (ms) of one launch: the callables in `launches` are
    captured back to back into one CUDA graph (programmatic dependent launch
    between them, as inside a decode step), the graph is replayed between two
    CUDA events on the replay stream, and the elapsed time is divided by the
    number of launches.  The mean over `reps` replays is returned."""
    import torch
    n = len(launches)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        for f in launches:
            f()
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            for f in launches:
                f()
    torch.cuda.current_stream().wait_stream(s)
    times = []
    with torch.cuda.stream(s):
        g.replay()  # warm
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            g.replay()
            b.record(s)
            b.synchronize()
            times.append(a.elapsed_time(b) / n)
    torch.cuda.synchronize()
    del g
    return statistics.mean(times)


class DecodeConfig3:
    """one decode token at position 4095 (KV context 4096)."""
    name = "decode-config3"
    unit = "tok/s"
    dtype = "u8/int32 (Q4_K/Q6_K x Q8_K), f32 decoder math"
    position = 4095
    k = 40

    def __init__(self):
        import torch

        from heliopause_b200 import synthetic as syn
        from heliopause_b200.model import CONFIG3, W_GATE, W_UP, CudaDecoderModel
        self.torch, self.syn = torch, syn
        self.shape = CONFIG3
        self.model = CudaDecoderModel(CONFIG3, max_tokens=8, top_k=64)
        self.model.load_gpu_synthetic(seed=1)
        self.model.fill_kv_random(self.position, seed=3)
        self.ids = torch.tensor([12345], dtype=torch.int32, device="cuda")
        self.pos = torch.tensor([self.position], dtype=torch.int32, device="cuda")
        self.vids = torch.tensor([12345, 7, 70000, 99, 4242], dtype=torch.int32, device="cuda")
        self.vpos = torch.tensor([self.position - 4 + i for i in range(5)], dtype=torch.int32, device="cuda")
        self.step_bytes = CONFIG3.weight_bytes() + CONFIG3.kv_read_bytes(self.position)
        self.launches_per_step = None
        self.W_GATE, self.W_UP = W_GATE, W_UP
        torch.cuda.synchronize()

    def step(self, ev=None):
        self.model.forward(self.ids, self.pos, self.k)

    def verify_step(self):
        self.model.forward(self.vids, self.vpos, self.k)

    def reordered_run(self, timed, steps: int) -> dict:
        """The same decode and verify steps on the reordered kernels
        (hpc_model_set_exact(0)): split-KV attention, fused norms, tensor-core
        GEMV for the verify width."""
        self.model.set_exact(False)
        try:
            self.model.fill_kv_random(self.position, seed=3)
            ms = timed(self.step, steps)
            vms = timed(self.verify_step, max(5, steps // 2))
        finally:
            self.model.set_exact(True)
            self.model.fill_kv_random(self.position, seed=3)
        return {"ms_per_step": ms, "tok_per_s": 1e3 / ms, "verify_ms_per_step": vms,
                "frac_of_hbm_peak": self.step_bytes / (ms / 1e3) / 1e9 / _peaks()["hbm_gbs"],
                "note": "reordered kernels (hpc_model_set_exact(0)): equal to the reference to f32 rounding, "
                        "amplified by the Q8_K re-quantization of every matmul input; the headline value is the "
                        "default, bit-exact step"}

    def e2e_step(self, host_ids):
        """Public API with host buffers: token id in, top-k ids/values out."""
        ids, vals = self.model.forward(host_ids, [self.position], self.k)
        ids.cpu()
        vals.cpu()

    def units_per_step(self) -> float:
        return 1.0

    def kernel_launch_count(self) -> int:
        s = self.shape
        # M = 1, hidden 2048, the default reference-order step (hc_model.cu
        # enqueue_step): the attention and FFN norms run inside the QKV and
        # gate/up GEMVs; per layer QKV, attention scores (with QK-norm / RoPE /
        # KV write), softmax, p.v, O, gate/up, GEGLU, down -- 285 launches at
        # 35 layers, as the ncu launch list of one step counts them
        per_layer = 8
        return 2 + s.layers * per_layer + 1 + 2  # rope rows + embed ... final norm + LM head + merge

    def roofline(self, peak_gbs: float) -> dict:
        """Dominant kernel: the gate/up GEMV (39% of the step's bytes), timed
        per launch over the model's 35 layers in one CUDA graph."""
        import ctypes as C

        from heliopause_b200 import _lib
        from heliopause_b200 import kernels as hk
        torch = self.torch
        L = _lib.lib()
        s = self.shape
        nbytes = C.c_size_t()
        L.hpc_q8_workspace_bytes(s.hidden, 1, C.byref(nbytes))
        ws = torch.zeros(nbytes.value, dtype=torch.uint8, device="cuda")
        x = torch.randn(s.hidden, device="cuda")
        hk.assert_cuda_ok(L.hpc_q8_quantize(C.c_void_p(x.data_ptr()), s.hidden, s.hidden, 1, C.c_void_p(ws.data_ptr()),
                                            nbytes.value, C.c_void_p(torch.cuda.current_stream().cuda_stream)), "q8")
        g = torch.empty(s.ffn, device="cuda")
        u = torch.empty(s.ffn, device="cuda")
        launches = []
        for layer in range(s.layers):
            hg = self.model.weight_handles[(layer, self.W_GATE)]
            hu = self.model.weight_handles[(layer, self.W_UP)]

            def f(hg=hg, hu=hu):
                hs = (C.c_void_p * 2)(hg.handle, hu.handle)
                outs = (C.c_void_p * 2)(g.data_ptr(), u.data_ptr())
                lens = (C.c_size_t * 2)(s.ffn, s.ffn)
                hk.assert_cuda_ok(L.hpc_matmul_q8(2, hs, C.c_void_p(ws.data_ptr()), nbytes.value, s.hidden, 1, outs,
                                                  lens, C.c_void_p(torch.cuda.current_stream().cuda_stream)), "gemv")
            launches.append(f)
        ms = graph_launch_times(launches)
        algo = 2 * self.syn.row_bytes(self.syn.Q4_K, s.hidden) * s.ffn + 4 * s.hidden + 8 * s.ffn
        achieved = algo / (ms / 1e3) / 1e9
        # the same launch as the step runs it: the post-attention residual and
        # the FFN RMSNorm computed by every CTA before it streams the weights
        # (hpc_matmul_rmsnorm_f32), 35 launches back to back with PDL
        xr = torch.randn(s.hidden, device="cuda")
        yr = torch.randn(s.hidden, device="cuda")
        wpost = torch.ones(s.hidden, device="cuda")
        wpre = torch.ones(s.hidden, device="cuda")
        xo = torch.empty(s.hidden, device="cuda")
        step_launches = []
        for layer in range(s.layers):
            hg = self.model.weight_handles[(layer, self.W_GATE)]
            hu = self.model.weight_handles[(layer, self.W_UP)]

            def f2(hg=hg, hu=hu):
                hs = (C.c_void_p * 2)(hg.handle, hu.handle)
                outs = (C.c_void_p * 2)(g.data_ptr(), u.data_ptr())
                lens = (C.c_size_t * 2)(s.ffn, s.ffn)
                hk.assert_cuda_ok(L.hpc_matmul_rmsnorm_f32(2, hs, C.c_void_p(ws.data_ptr()), nbytes.value, s.hidden, 1,
                                                           C.c_void_p(xr.data_ptr()), C.c_void_p(yr.data_ptr()),
                                                           C.c_void_p(wpost.data_ptr()), C.c_void_p(wpre.data_ptr()),
                                                           1e-6, C.c_void_p(xo.data_ptr()), outs, lens,
                                                           C.c_void_p(torch.cuda.current_stream().cuda_stream)),
                                  "gemv + norm prologue")
            step_launches.append(f2)
        ms_step = graph_launch_times(step_launches)
        achieved_step = algo / (ms_step / 1e3) / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s", "frac": achieved / peak_gbs,
                "traffic": None, "kernel": "hc_gemvw_kernel<1> (ffn gate+up, 2048 -> 2x16384 Q4_K, M=1, reference "
                                           "f32 order, input pre-quantized: hpc_matmul_q8)",
                "algorithmic_bytes_per_launch": algo, "launch_ms": ms,
                "in_step": {"kernel": "the same launch with the step's fused prologue (residual add, two RMSNorms, "
                                      "Q8_K in every CTA: hpc_matmul_rmsnorm_f32), as the default step runs it",
                            "launch_ms": ms_step, "achieved": achieved_step, "frac": achieved_step / peak_gbs}}

    def config(self) -> dict:
        s = self.shape
        return {"workload": "decode one token, E4B-shaped Q4_K_M decoder (BASELINE config 3)",
                "order": "reference f32 order (bit-exact to the oracle)",
                "layers": s.layers, "hidden": s.hidden, "heads": s.heads, "kv_heads": s.kv_heads,
                "head_dim": s.head_dim, "ffn": s.ffn, "vocab": s.vocab, "kv_layers": s.kv_layers,
                "context": s.context, "position": self.position, "top_k": self.k, "kv_dtype": "f32",
                "bytes_per_token": self.step_bytes,
                "l2": f"inputs larger than L2: {self.step_bytes / 1e9:.2f} GB of weights+KV streamed per step"}

    def mtp_run(self, n_tokens: int = 256, n_spec: int = 4, context: int = 1024) -> dict:
        """MTP speculative decoding on this model -- a
        one-layer draft head of the same width proposes n_spec tokens, one
        batched verify over n_spec + 1 positions, sampling acceptance at
        temperature 1 with seeded uniforms, n_tokens generated from position
        `context`.  Wall clock of the whole host loop (draft, verify, accept)."""
        import time as _t

        from heliopause_b200 import generation as gen
        from heliopause_b200.mtp import CudaMtpDraftHead, MtpDraftShape, MtpGenerator, SyntheticDraftWeights
        torch = self.torch
        ds = MtpDraftShape()
        head = CudaMtpDraftHead(ds, SyntheticDraftWeights(ds, seed=7), gpu_seed=7)
        g = MtpGenerator(self.model, head)
        opt = gen.resolve_generation_sampling_options(do_sample=True, temperature=1.0, seed=1234)
        rng = gen.create_deterministic_rng(opt.seed)
        first, ctx = g.start(12345, context - 1, opt, rng)  # warms the draft/verify paths' buffers
        g.generate(first, ctx, 8, n_spec, opt, rng)
        rng = gen.create_deterministic_rng(opt.seed)
        torch.cuda.synchronize()
        t0 = _t.perf_counter()
        first, ctx = g.start(12345, context - 1, opt, rng)
        toks, rounds, acc = g.generate(first, ctx, n_tokens, n_spec, opt, rng)
        torch.cuda.synchronize()
        dt = _t.perf_counter() - t0
        # one draft step on its own (device time of the step's graph and copies)
        kv = [self.model.kv(layer) for layer in g.kv_layers]
        emb, hid = g.embedding(12345), ctx.current_hidden
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        head.run(emb, hid, kv, ctx.position, 64)
        a.record()
        for _ in range(20):
            head.run(emb, hid, kv, ctx.position, 64)
        b.record()
        torch.cuda.synchronize()
        draft_ms = a.elapsed_time(b) / 20
        head.close()
        del g, head
        torch.cuda.empty_cache()
        return {"tokens": len(toks), "tok_per_s": len(toks) / dt, "seconds": dt, "rounds": rounds,
                "accepted_drafts": acc, "acceptance_rate": acc / max(1, rounds * n_spec),
                "draft_tokens_per_round": n_spec, "context_start": context, "draft_step_ms": draft_ms,
                "sampling": {"temperature": opt.temperature, "top_k": opt.top_k, "top_p": opt.top_p, "seed": opt.seed},
                "note": "config 4: random draft-head weights (acceptance near chance); draft head = hpc_draft_step "
                        "(dequant-fused matmuls over the head's resident quantized tiles, one CUDA graph per step), "
                        "verify = the fused decoder forward at "
                        "M=n_spec+1; tok_per_s is the wall clock of the host loop (drafts drawn on the device: one host "
                        "synchronization per round, after the verify)"}

    @classmethod
    def cpu_sampler(cls, threads: int):
        return CpuDecodeSample(threads, cls.position, cls.k)

    def cpu_baseline(self, budget_s: float, threads: int) -> dict:
        return cpu_baseline_from(self.cpu_sampler(threads), budget_s)


class CpuDecodeSample:
    """The C restatement of the WASM decode path on the host cores: a bounded
    sample of 2 full decoder layers at context 4096 (one writing KV) plus the
    262,144-row LM head and top-40, scaled to the model's 35 layers."""

    def __init__(self, threads: int, position: int, k: int):
        from heliopause_b200.model import CONFIG3, SyntheticWeights
        from oracle.decoder_oracle import OracleDecoder
        self.s = CONFIG3
        self.threads, self.position, self.k = threads, position, k
        self.w = SyntheticWeights(CONFIG3, seed=1)
        self.ref = OracleDecoder(CONFIG3, self.w, threads=threads)
        kc, vc = self.w.kv(0, position)
        self.ref.set_kv(0, kc, vc)
        self.ref.set_kv(1, kc.copy(), vc.copy())
        self.x0 = self.ref.embed([12345])
        self.ref._lm_head()
        self.ref._weight(0, 0)

    def run(self) -> tuple[float, float]:
        """Seconds for (2 layers, LM head + top-k)."""
        from oracle import oracle as o
        s = self.s
        t0 = time.perf_counter()
        x = self.x0
        for layer in (0, 1):
            x = self.ref.layer(layer, x, [self.position])
        t_layers = time.perf_counter() - t0
        data, scales = self.ref._lm_head()
        norm = o.rms_norm_rows(x, self.w.output_norm(), s.rms_eps)
        t1 = time.perf_counter()
        logits = o.matmul_prepared(o.Q6_K, data, scales, norm, s.hidden, s.vocab, 1, threads=self.threads)
        o.topk(logits, self.k)
        return t_layers, time.perf_counter() - t1

    def per_token(self, t_layers: float, t_head: float) -> float:
        return t_layers / 2 * self.s.layers + t_head

    def describe(self, t_layers: float, t_head: float) -> str:
        return (f"2 decoder layers at context {self.s.context} ({t_layers:.2f} s) + LM head/top-{self.k} "
                f"({t_head:.2f} s) of the C restatement of the WASM path on {self.threads} threads, "
                f"scaled to {self.s.layers} layers")


def cpu_baseline_from(sampler, budget_s: float) -> dict:
    sampler.run()  # warm
    t0 = time.perf_counter()
    runs = []
    while True:
        runs.append(sampler.run())
        if time.perf_counter() - t0 >= budget_s:
            break
    tl = statistics.median(r[0] for r in runs)
    th = statistics.median(r[1] for r in runs)
    return {"value": 1.0 / sampler.per_token(tl, th), "unit": "tok/s", "cores": sampler.threads, "kind": "port",
            "sample": f"{len(runs)} x (" + sampler.describe(tl, th) + ")"}


class _Q8Launcher:
    """Raw C-ABI launches on a caller-owned Q8_K workspace (the graph-capturable
    form the decode step uses): hpc_q8_quantize + hpc_matmul_q8."""

    def __init__(self, k: int, m: int):
        import ctypes as C

        import torch

        from heliopause_b200 import _lib
        from heliopause_b200 import kernels as hk
        self.C, self.L, self.hk, self.torch = C, _lib.lib(), hk, torch
        self.k, self.m = k, m
        nbytes = C.c_size_t()
        hk.assert_cuda_ok(self.L.hpc_q8_workspace_bytes(k, m, C.byref(nbytes)), "workspace bytes")
        self.ws_bytes = nbytes.value
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device="cuda")

    def stream(self):
        return self.C.c_void_p(self.torch.cuda.current_stream().cuda_stream)

    def quantize(self, x):
        self.hk.assert_cuda_ok(self.L.hpc_q8_quantize(self.C.c_void_p(x.data_ptr()), x.numel(), self.k, self.m,
                                                      self.C.c_void_p(self.ws.data_ptr()), self.ws_bytes,
                                                      self.stream()), "q8")

    def matmul(self, handles, outs):
        C = self.C
        n = len(handles)
        hs = (C.c_void_p * n)(*[h.handle for h in handles])
        ps = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
        ls = (C.c_size_t * n)(*[o.numel() for o in outs])
        self.hk.assert_cuda_ok(self.L.hpc_matmul_q8(n, hs, C.c_void_p(self.ws.data_ptr()), self.ws_bytes, self.k,
                                                    self.m, ps, ls, self.stream()), "gemv")


class GemvConfig2:
    """the projections of one decoder layer, launched as the
    decode step launches them: [Q, K, V] (one launch on one Q8_K input),
    [gate, up] (one launch), and the Q6_K down projection.  M = --cols."""
    name = "gemv-config2"
    unit = "GB/s"
    dtype = "u8"
    K, F = 2048, 16384
    copies = 4

    def __init__(self, m: int = 1):
        import torch

        from heliopause_b200 import kernels as hk
        from heliopause_b200 import synthetic as syn
        self.torch, self.hk, self.syn, self.M = torch, hk, syn, m
        K, F = self.K, self.F
        shapes = [("Q4_K", K, 2048), ("Q4_K", K, 512), ("Q4_K", K, 512), ("Q4_K", K, F), ("Q4_K", K, F),
                  ("Q6_K", F, K)]
        self.sets = []
        for c in range(self.copies):
            hs = [hk.create_quantized_weight_handle(t, syn.quant_weight(syn.Q4_K if t == "Q4_K" else syn.Q6_K, n, k,
                                                                        seed=2000 + 10 * c + i), k, n)
                  for i, (t, k, n) in enumerate(shapes)]
            self.sets.append(hs)
        self.w_bytes = sum(syn.row_bytes(syn.Q4_K if t == "Q4_K" else syn.Q6_K, k) * n for t, k, n in shapes)
        self.algo_bytes = self.w_bytes + 4 * m * (K + F) + 4 * m * (2048 + 512 + 512 + 2 * F + K)
        self.qin = _Q8Launcher(K, m)
        self.qdown = _Q8Launcher(F, m)
        self.x = torch.from_numpy(syn.activations(m, K, seed=7)).cuda()
        self.a = torch.from_numpy(syn.activations(m, F, seed=8)).cuda()
        self.outs = [torch.empty(n * m, device="cuda") for _, _, n in shapes]
        self.i = 0

    def step(self, ev=None):
        hs = self.sets[self.i % self.copies]
        self.i += 1
        self.qin.quantize(self.x)
        self.qin.matmul(hs[0:3], self.outs[0:3])
        self.qin.matmul(hs[3:5], self.outs[3:5])
        self.qdown.quantize(self.a)
        self.qdown.matmul(hs[5:6], self.outs[5:6])

    def e2e_step(self, host_x):
        hs = self.sets[self.i % self.copies]
        self.i += 1
        for h, n in ((hs[0], 2048), (hs[3], self.F)):
            self.hk.mat_mul_quantized_resident(h, host_x, self.K, n, self.M)  # host in -> host out

    def host_input(self):
        return self.syn.activations(self.M, self.K, seed=7), 4 * self.K * self.M, 4 * (2048 + self.F) * self.M

    def units_per_step(self) -> float:
        return self.algo_bytes / 1e9

    def kernel_launch_count(self) -> int:
        return 5

    def roofline(self, peak_gbs: float) -> dict:
        hs = [s[3:5] for s in self.sets]
        launches = [lambda h=h: self.qin.matmul(h, self.outs[3:5]) for h in hs]
        ms = graph_launch_times(launches * 2)
        algo = 2 * self.syn.row_bytes(self.syn.Q4_K, self.K) * self.F + 4 * self.K * self.M + 8 * self.F * self.M
        achieved = algo / (ms / 1e3) / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s", "frac": achieved / peak_gbs,
                "traffic": None, "kernel": f"hc_gemvw_kernel (gate+up, 2048 -> 2x16384 Q4_K, M={self.M}, reference f32 order)",
                "algorithmic_bytes_per_launch": algo, "launch_ms": ms}

    def config(self) -> dict:
        return {"workload": f"config-2 projections (QKV | gate+up | Q6_K down), M={self.M} (BASELINE config 2)",
                "K": self.K, "ffn": self.F, "M": self.M, "weight_copies_rotated": self.copies,
                "l2": f"inputs larger than L2: {self.copies} weight sets = "
                      f"{self.copies * self.w_bytes / 1e6:.0f} MB rotated per step"}

    def cpu_baseline(self, budget_s: float, threads: int) -> dict:
        return None


class LmHeadConfig5:
    """BASELINE config 5 (single GPU, M = --cols): Q6_K LM head 2048 -> 262,144
    fused with top-40 (q8 quantize, GEMV + candidate lists, merge)."""
    name = "lmhead-config5"
    unit = "GB/s"
    dtype = "u8"
    K, V, TOPK = 2048, 262144, 40

    def __init__(self, m: int = 1):
        import ctypes as C

        import torch

        from heliopause_b200 import kernels as hk
        from heliopause_b200 import synthetic as syn
        self.torch, self.hk, self.syn, self.C, self.M = torch, hk, syn, C, m
        world, rank, _ = _dist()
        self.world = world
        self.scaling = "strong" if world > 1 else "weak"
        full = syn.q6_k_weight(self.V, self.K, seed=3000)
        self.w_bytes = syn.row_bytes(syn.Q6_K, self.K) * self.V
        if world > 1:
            # vocabulary rows split over the ranks; keys all-gathered over NCCL
            from heliopause_b200 import sharded_head as sh
            first, n = sh.shard_rows(self.V, world)[rank]
            rb = syn.row_bytes(syn.Q6_K, self.K)
            self.backend = sh.CudaShardBackend("Q6_K", full[first * rb:(first + n) * rb], self.K, n, first, m,
                                               self.TOPK)
            self.sharded = sh.ShardedLmHead(self.backend, self.TOPK)
            self.x = torch.from_numpy(syn.activations(m, self.K, seed=9)).cuda()
            self.algo_bytes = self.w_bytes + 4 * self.K * m + 8 * self.TOPK * m
            self.head = self.backend.handle
            return
        self.head = hk.create_quantized_weight_handle("Q6_K", full, self.K, self.V)
        self.algo_bytes = self.w_bytes + 4 * self.K * m + 8 * self.TOPK * m
        self.q = _Q8Launcher(self.K, m)
        cb = C.c_size_t()
        hk.assert_cuda_ok(self.q.L.hpc_lm_head_candidates_bytes(self.head.handle, m, self.TOPK, C.byref(cb)), "cand")
        self.cand_bytes = cb.value
        self.cand = torch.empty(self.cand_bytes, dtype=torch.uint8, device="cuda")
        self.x = torch.from_numpy(syn.activations(m, self.K, seed=9)).cuda()
        self.ids = torch.empty(m * self.TOPK, dtype=torch.int32, device="cuda")
        self.vals = torch.empty(m * self.TOPK, device="cuda")

    def head_launch(self):
        C, q = self.C, self.q
        self.hk.assert_cuda_ok(q.L.hpc_lm_head_topk_q8(
            self.head.handle, C.c_void_p(q.ws.data_ptr()), q.ws_bytes, self.K, self.M, self.TOPK, 0,
            C.c_void_p(self.cand.data_ptr()), self.cand_bytes, C.c_float(0.0), C.c_void_p(self.ids.data_ptr()),
            C.c_void_p(self.vals.data_ptr()), None, q.stream()), "lm head")

    def step(self, ev=None):
        if self.world > 1:
            self.sharded.topk(self.x, self.M)
            return
        self.q.quantize(self.x)
        self.head_launch()

    def e2e_step(self, host_x):
        if self.world > 1:
            ids, vals = self.sharded.topk(host_x.to("cuda", non_blocking=True), self.M)
        else:
            ids, vals = self.hk.lm_head_topk(self.head, host_x, self.M, self.TOPK)
        ids.cpu()
        vals.cpu()

    def host_input(self):
        return self.syn.activations(self.M, self.K, seed=9), 4 * self.K * self.M, 8 * self.TOPK * self.M

    def units_per_step(self) -> float:
        return self.algo_bytes / 1e9

    def kernel_launch_count(self) -> int:
        return 4 if self.world > 1 else 3

    def roofline(self, peak_gbs: float) -> dict:
        if self.world > 1:
            return {"bound": "hbm", "achieved": None, "peak": peak_gbs, "unit": "GB/s", "frac": None,
                    "traffic": None, "kernel": "row-sharded head: per-rank roofline is the 1-GPU line"}
        self.q.quantize(self.x)
        ms = graph_launch_times([self.head_launch] * 4)
        achieved = self.algo_bytes / (ms / 1e3) / 1e9
        return {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s", "frac": achieved / peak_gbs,
                "traffic": None, "kernel": f"hc_lmhead_topk_kernel<{self.M}> + hc_topk_merge_kernel (Q6_K 2048 -> 262144, "
                                           f"top-{self.TOPK}, M={self.M})",
                "algorithmic_bytes_per_launch": self.algo_bytes, "launch_ms": ms}

    def config(self) -> dict:
        return {"workload": f"Q6_K LM head 2048 -> 262144 + top-40, M={self.M} (BASELINE config 5, one GPU)",
                "K": self.K, "vocab": self.V, "M": self.M, "top_k": self.TOPK,
                "l2": f"inputs larger than L2: {self.w_bytes / 1e6:.0f} MB of weights per step"}

    def cpu_baseline(self, budget_s: float, threads: int) -> dict:
        return None


class PrefillConfig5:
    """BASELINE config 5 prefill: 512 tokens of N(0,1) hidden through the
    config-3 stack (hpc_model_prefill): tensor-core (mma.sync s8) matmuls at
    M = 512 and causal attention over the prompt."""
    name = "prefill-config5"
    unit = "tok/s"
    dtype = "u8/int32 (Q4_K/Q6_K x Q8_K, s8 tensor-core mma), f32 decoder math"
    N = 512

    def __init__(self):
        import torch

        from heliopause_b200 import synthetic as syn
        from heliopause_b200.model import CONFIG3, W_GATE, W_UP, CudaDecoderModel
        self.torch, self.syn, self.shape = torch, syn, CONFIG3
        self.model = CudaDecoderModel(CONFIG3, max_tokens=8, top_k=64)
        self.model.load_gpu_synthetic(seed=1)
        g = torch.Generator(device="cuda")
        g.manual_seed(5)
        self.x = torch.randn(self.N, CONFIG3.hidden, device="cuda", generator=g)
        self.W_GATE, self.W_UP = W_GATE, W_UP
        s = CONFIG3
        wcount = 0
        for layer in range(s.layers):
            for slot in s.slots(layer):
                k, r = s.weight_shape(slot)
                wcount += k * r
        # matmul MACs + causal attention (QK and PV over on average N/2 keys)
        self.flops = 2.0 * self.N * wcount + 2.0 * 2 * s.layers * s.heads * s.head_dim * self.N * (self.N + 1) / 2
        self.model.prefill(self.x, 0)
        torch.cuda.synchronize()

    def step(self, ev=None):
        self.model.prefill(self.x, 0)

    def e2e_step(self, host_x):
        self.model.prefill(host_x, 0).cpu()

    def host_input(self):
        x = self.syn.rng(5).standard_normal((self.N, self.shape.hidden)).astype("float32")
        return x, x.nbytes, x.nbytes

    def units_per_step(self) -> float:
        return float(self.N)

    def kernel_launch_count(self) -> int:
        s = self.shape
        own, shared = s.kv_layers, s.layers - s.kv_layers
        # norm, Q/K/V, qk-post, attention, O, norm, gate, up, geglu, down (shared-KV layers: Q only)
        return 1 + own * 12 + shared * 10 + 1

    def roofline(self, peak_gbs: float) -> dict:
        """Dominant kernel: the gate/up matmul at M = 512 (34% of the FLOPs),
        35 launches (one per layer's weights) back to back in a graph."""
        import ctypes as C

        from heliopause_b200 import _lib
        from heliopause_b200 import kernels as hk
        torch, s = self.torch, self.shape
        L = _lib.lib()
        nbytes = C.c_size_t()
        L.hpc_q8_workspace_bytes(s.hidden, self.N, C.byref(nbytes))
        ws = torch.zeros(nbytes.value, dtype=torch.uint8, device="cuda")
        st = lambda: C.c_void_p(torch.cuda.current_stream().cuda_stream)
        hk.assert_cuda_ok(L.hpc_q8_quantize(C.c_void_p(self.x.data_ptr()), self.x.numel(), s.hidden, self.N,
                                            C.c_void_p(ws.data_ptr()), nbytes.value, st()), "q8")
        g = torch.empty(self.N * s.ffn, device="cuda")
        u = torch.empty(self.N * s.ffn, device="cuda")
        launches = []
        for layer in range(s.layers):
            hg = self.model.weight_handles[(layer, self.W_GATE)]
            hu = self.model.weight_handles[(layer, self.W_UP)]

            def f(hg=hg, hu=hu):
                hs = (C.c_void_p * 2)(hg.handle, hu.handle)
                outs = (C.c_void_p * 2)(g.data_ptr(), u.data_ptr())
                lens = (C.c_size_t * 2)(self.N * s.ffn, self.N * s.ffn)
                hk.assert_cuda_ok(L.hpc_matmul_q8(2, hs, C.c_void_p(ws.data_ptr()), nbytes.value, s.hidden, self.N,
                                                  outs, lens, st()), "gemm")
            launches.append(f)
        ms = graph_launch_times(launches)
        flops = 2.0 * self.N * s.hidden * 2 * s.ffn
        achieved = flops / (ms / 1e3) / 1e12
        peaks = _peaks()
        peak = peaks.get("bf16_tflops") or 1590.0
        return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "traffic": None, "kernel": "hc_gemm_tc_kernel<Q4_K> x2 (ffn gate+up, 2048 -> 2x16384, M=512)",
                "peak_note": "measured dense bf16 cuBLAS peak; the kernel computes s8 x s8 -> s32 on mma.sync",
                "flops_per_launch": flops, "launch_ms": ms}

    def config(self) -> dict:
        s = self.shape
        return {"workload": "prefill 512 tokens through the config-3 stack (BASELINE config 5)", "tokens": self.N,
                "layers": s.layers, "hidden": s.hidden, "ffn": s.ffn, "positions": "0..511",
                "flops_per_step": self.flops, "l2": "2.3 GB of weights per step, larger than L2"}

    def cpu_baseline(self, budget_s: float, threads: int) -> dict:
        """The oracle's layer (C restatement) for 8 tokens of one config-3
        layer, scaled to 35 layers."""
        import numpy as np

        from heliopause_b200.model import SyntheticWeights
        from oracle.decoder_oracle import OracleDecoder
        s = self.shape
        ref = OracleDecoder(s, SyntheticWeights(s, 1), threads=threads)
        ref.set_kv(0, np.zeros((s.context, s.kv_heads, s.head_dim), np.float32),
                   np.zeros((s.head_dim, s.kv_heads, s.context), np.float32))
        x = self.syn.rng(5).standard_normal((8, s.hidden)).astype(np.float32).reshape(-1)
        ref.layer(0, x, list(range(8)))  # warm the prepared-scale cache
        t0 = time.perf_counter()
        runs = 0
        while True:
            ref.layer(0, x, list(range(8)))
            runs += 1
            if time.perf_counter() - t0 >= budget_s:
                break
        per_layer = (time.perf_counter() - t0) / runs
        return {"value": 8.0 / (per_layer * s.layers), "unit": "tok/s", "cores": threads, "kind": "port",
                "sample": f"{runs} x one config-3 layer over 8 prompt tokens ({per_layer:.2f} s each) on {threads} "
                          f"threads, scaled to {s.layers} layers"}


def sharded_lm_head_run(world: int, rank: int, steps: int, warmup: int) -> dict:
    """The row-sharded Q6_K LM head 2048 -> 262,144 + top-40 over every rank
    (BASELINE config 5 / the multi-GPU row of the scope table): each rank holds
    its contiguous vocabulary slice, runs the fused GEMV + top-k with its
    first row as the id offset, the 64-bit keys are all-gathered over NCCL and
    every rank merges them (heliopause_b200/sharded_head.py).  For M = 1, 5
    and 64 columns: device time per call (CUDA events, max over ranks), the
    time of the local slice alone, and hence the all-gather + merge share.
    Rank 0 checks the merged ids and values against the unsharded
    hpc_lm_head_topk on the whole head."""
    import torch
    import torch.distributed as dist

    from heliopause_b200 import kernels as hk
    from heliopause_b200 import sharded_head as sh
    from heliopause_b200 import synthetic as syn
    K, V, k = 2048, 262144, 40
    full = syn.q6_k_weight(V, K, seed=3000)
    first, n = sh.shard_rows(V, world)[rank]
    rb = syn.row_bytes(syn.Q6_K, K)
    backend = sh.CudaShardBackend("Q6_K", full[first * rb:(first + n) * rb], K, n, first, 64, k)
    head = sh.ShardedLmHead(backend, k)
    whole = hk.create_quantized_weight_handle("Q6_K", full, K, V) if rank == 0 else None
    del full

    def device_ms(fn, count):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(count):
            fn()
        b.record()
        torch.cuda.synchronize()
        dist.barrier()
        t = torch.tensor([a.elapsed_time(b) / count], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0])

    out = {"vocab": V, "hidden": K, "top_k": k, "ranks": world, "rows_per_rank": n, "scaling": "strong",
           "collective": "all_gather_into_tensor of k*M int64 keys per rank (NCCL), then hpc_topk_merge_keys",
           "per_m": []}
    count = max(10, min(steps, 50))
    for m in (1, 5, 64):
        x = torch.from_numpy(syn.activations(m, K, seed=9 + m)).cuda()
        total = device_ms(lambda: head.topk(x, m), count)
        local = device_ms(lambda: backend.local_keys(x, m), count)
        ids, vals = head.topk(x, m)
        entry = {"m": m, "ms_per_call": total, "local_slice_ms": local,
                 "gather_merge_ms": max(0.0, total - local), "gather_merge_share": max(0.0, total - local) / total,
                 "columns_per_s": m / (total / 1e3),
                 "weight_gbs_per_rank": syn.row_bytes(syn.Q6_K, K) * n / (local / 1e3) / 1e9}
        if rank == 0:
            rid, rval = hk.lm_head_topk(whole, x, m, k)
            gi, gv = ids.reshape(m, k).cpu(), vals.reshape(m, k).cpu()
            ri, rv = rid.reshape(m, k).cpu(), rval.reshape(m, k).cpu()
            entry["ids_equal_unsharded"] = bool(torch.equal(gi, ri))
            entry["values_equal_unsharded"] = bool(torch.equal(gv, rv))
        out["per_m"].append(entry)
    if whole is not None:
        hk.release_quantized_weight_handle(whole)
    backend.release()
    torch.cuda.synchronize()
    dist.barrier()
    return out


WORKLOADS = {"decode-config3": DecodeConfig3, "gemv-config1": GemvConfig1, "gemv-config2": GemvConfig2,
             "lmhead-config5": LmHeadConfig5, "prefill-config5": PrefillConfig5}


# ------------------------------------------------------------------- main ---

def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args, world, rank):
    """CPU reference arm (rank 0 only): the C restatement of the reference's
    WASM path (the reference itself cannot run here) on all host threads."""
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0))
    if args.workload == "decode-config3":
        sampler = DecodeConfig3.cpu_sampler(threads)
        for _ in range(args.warmup):
            sampler.run()
        t0 = time.perf_counter()
        runs = [sampler.run() for _ in range(args.steps)]
        elapsed = time.perf_counter() - t0
        tl = statistics.median(r[0] for r in runs)
        th = statistics.median(r[1] for r in runs)
        v = 1.0 / sampler.per_token(tl, th)
        cfg = {"workload": "decode one token, E4B-shaped Q4_K_M decoder (BASELINE config 3)", "context": 4096,
               "position": DecodeConfig3.position, "top_k": DecodeConfig3.k}
        cb = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port",
              "sample": "each step: " + sampler.describe(tl, th)}
        unit, dtype = "tok/s", DecodeConfig3.dtype
    else:
        wl = GemvConfig1.__new__(GemvConfig1)
        import heliopause_b200.synthetic as syn
        wl.syn = syn
        wl.w_bytes = syn.row_bytes(syn.Q4_K, wl.K) * wl.N
        wl.algo_bytes = wl.w_bytes + 4 * wl.K * wl.M + 4 * wl.N * wl.M
        budget = max(1.0, 60.0 / max(1, args.steps + args.warmup))
        for _ in range(args.warmup):
            wl.cpu_baseline(0.0, threads)
        t0 = time.perf_counter()
        vals = [wl.cpu_baseline(budget, threads) for _ in range(args.steps)]
        elapsed = time.perf_counter() - t0
        v = statistics.median(x["value"] for x in vals)
        cb = dict(vals[-1])
        cb["value"] = v
        cfg = wl.config()
        unit, dtype = wl.unit, wl.dtype
    line = {"metric": METRIC, "value": v, "unit": unit, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed * 1e3 / max(1, args.steps),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
            "data": "synthetic (seeded, BASELINE distributions)", "config": cfg, "cpu_baseline": cb,
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="decode-config3")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-mtp", action="store_true", help="skip the config-4 MTP generation field")
    ap.add_argument("--cols", type=int, default=1,
                    help="columns (tokens) for the gemv-config2 / lmhead-config5 workloads")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = _dist()

    if args.impl == "reference":
        run_reference(args, world, rank)
        return

    import torch
    import torch.distributed as dist

    from heliopause_b200 import kernels as hk

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    hk.init_device(local)
    wl = WORKLOADS[args.workload](args.cols) if args.workload in ("gemv-config2", "lmhead-config5") \
        else WORKLOADS[args.workload]()

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(fn, steps):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / steps], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0])

    with ClockSampler(local) as clk:
        ms = timed(wl.step, args.steps)
    # weak scaling: every rank processes its own step; strong: one step's work is split over the ranks
    ranks_of_work = world if getattr(wl, "scaling", "weak") == "weak" else 1
    value = wl.units_per_step() * ranks_of_work / (ms / 1e3)

    verify = None
    if hasattr(wl, "verify_step"):
        vms = timed(wl.verify_step, max(5, args.steps // 2))
        verify = {"m": 5, "ms_per_step": vms, "positions_per_s": 5 * world / (vms / 1e3),
                  "note": "one batched forward over 5 positions (MTP verify width), top-40 per position"}
    reordered = wl.reordered_run(timed, args.steps) if hasattr(wl, "reordered_run") else None

    # end to end through the public API with host buffers
    if args.workload == "decode-config3":
        host_in = torch.tensor([12345], dtype=torch.int32).pin_memory()
        h2d, d2h = 8, 8 * wl.k
    elif hasattr(wl, "host_input"):
        hx, h2d, d2h = wl.host_input()
        host_in = torch.from_numpy(hx).pin_memory()
    else:
        host_in = torch.from_numpy(wl.syn.activations(wl.M, wl.K, seed=7)).pin_memory()
        h2d, d2h = 4 * wl.K * wl.M, 4 * wl.N * wl.M
    for _ in range(3):
        wl.e2e_step(host_in)
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    n_e2e = max(5, args.steps // 2)
    for _ in range(n_e2e):
        wl.e2e_step(host_in)
    torch.cuda.synchronize()
    e2e_s = torch.tensor([(time.perf_counter() - t0) / n_e2e], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    e2e_value = wl.units_per_step() * ranks_of_work / float(e2e_s[0])

    mtp = wl.mtp_run() if hasattr(wl, "mtp_run") and not args.no_mtp and world == 1 else None
    sharded = sharded_lm_head_run(world, rank, args.steps, args.warmup) \
        if world > 1 and args.workload == "decode-config3" else None

    peaks = _peaks()
    roofline = wl.roofline(peaks["hbm_gbs"])
    roofline["peak_source"] = peaks["source"]
    prof = ROOT / "profiles" / "traffic.json"
    if prof.exists():
        tr = json.loads(prof.read_text()).get(wl.name)
        if tr and getattr(wl, "M", 1) == 1 and world == 1:  # the captures are 1-GPU, M=1 launches
            roofline["traffic"] = tr

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = len(os.sched_getaffinity(0))
        cpu = wl.cpu_baseline(10.0, threads)
        # the reference's own default pool size: "auto" = min(8, max(1, floor(cores / 2)))
        # (runner/wasm/acceleration.ts:277-283)
        auto = min(8, max(1, threads // 2))
        if cpu is not None and auto != threads:
            d = wl.cpu_baseline(10.0, auto)
            cpu["reference_default_threads"] = {"cores": auto, "value": d["value"], "unit": d["unit"],
                                                "rule": "min(8, max(1, floor(cores/2))), acceleration.ts:277-283",
                                                "sample": d["sample"]}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": wl.unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": getattr(wl, "scaling", "weak"), "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded, BASELINE distributions)",
                "config": wl.config(), "roofline": roofline, "cpu_baseline": cpu,
                "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
                "gpu_launches": wl.kernel_launch_count() * args.steps, "clocks": clk.summary()}
        if hasattr(wl, "step_bytes"):
            line["step_hbm"] = {"bytes_per_step": wl.step_bytes,
                                "achieved_gbs": wl.step_bytes / (ms / 1e3) / 1e9,
                                "frac_of_peak": wl.step_bytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]}
        if verify:
            line["verify"] = verify
        if reordered:
            line["reordered"] = reordered
        if mtp:
            line["mtp"] = mtp
        if sharded:
            line["sharded_lm_head"] = sharded
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
