"""Benchmark for the Heliopause decode hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Prints ONE JSON line (rank 0).  For N > 1 launch under torchrun; each rank
runs its own replica/shard and the reported time is the max over ranks.

Workloads (a "step" is one pass of the hot path over one batch of synthetic
input, inputs resident in HBM when the timed region starts):
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
        self.t = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
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
        for ln in self.lines:
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


WORKLOADS = {"gemv-config1": GemvConfig1}


# ------------------------------------------------------------------- main ---

def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args, world, rank):
    """CPU reference arm (rank 0 only)."""
    if rank != 0:
        return
    wl_cls = WORKLOADS[args.workload]
    threads = os.cpu_count() or 1
    try:
        threads = len(os.sched_getaffinity(0))
    except AttributeError:
        pass
    wl = wl_cls.__new__(wl_cls)
    import heliopause_b200.synthetic as syn
    wl.syn = syn
    wl.w_bytes = syn.row_bytes(syn.Q4_K, wl.K) * wl.N
    wl.algo_bytes = wl.w_bytes + 4 * wl.K * wl.M + 4 * wl.N * wl.M
    budget = max(2.0, 60.0 / max(1, args.steps + args.warmup))
    for _ in range(args.warmup):
        wl.cpu_baseline(0.0, threads)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        vals.append(wl.cpu_baseline(budget, threads))
    elapsed = time.perf_counter() - t0
    v = statistics.median(x["value"] for x in vals)
    cb = dict(vals[-1])
    cb["value"] = v
    line = {"metric": METRIC, "value": v, "unit": wl.unit, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed * 1e3 / max(1, args.steps),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": wl.dtype,
            "data": "synthetic (seeded PCG64, BASELINE distributions)", "config": wl.config(),
            "cpu_baseline": cb, "e2e": {"value": v, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="gemv-config1")
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
    wl = WORKLOADS[args.workload]()

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        wl.step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        start.record()
        for i in range(args.steps):
            wl.step(kev[i])
        end.record()
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    t = torch.tensor([ms, kern_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, kern_ms = float(t[0]), float(t[1])
    value = wl.units_per_step() * world / (ms / 1e3)

    # end to end through the public API with host buffers (pinned input)
    host_x = torch.from_numpy(wl.syn.activations(wl.M, wl.K, seed=7)).pin_memory()
    for _ in range(3):
        wl.e2e_step(host_x)
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        wl.e2e_step(host_x)
    torch.cuda.synchronize()
    e2e_s = torch.tensor([(time.perf_counter() - t0) / args.steps], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
    e2e_value = wl.units_per_step() * world / float(e2e_s[0])

    peaks = _peaks()
    achieved = wl.algo_bytes / (kern_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                "kernel": "gemv_kernel<1>", "peak_source": peaks["source"]}
    prof = ROOT / "profiles" / "traffic.json"
    if prof.exists():
        tr = json.loads(prof.read_text()).get(wl.name)
        if tr:
            roofline["traffic"] = tr

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = len(os.sched_getaffinity(0))
        cpu = wl.cpu_baseline(10.0, threads)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": wl.unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic (seeded PCG64, BASELINE distributions)",
                "config": wl.config(), "roofline": roofline, "cpu_baseline": cpu,
                "e2e": {"value": e2e_value, "unit": wl.unit, "h2d_bytes_per_step": 4 * wl.K * wl.M,
                        "d2h_bytes_per_step": 4 * wl.N * wl.M},
                "gpu_launches": wl.launches_per_step * args.steps, "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
