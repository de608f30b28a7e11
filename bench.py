#!/usr/bin/env python
"""Benchmark of the B200 kernels behind stable-diffusion.assembly's hook surface.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1); every rank runs the same workload on
its own GPU (replicas: weak scaling, no data-path collective), the step time
is the max over ranks, and rank 0 prints one JSON line.

The step (workload "sd15_hot_ops"): the hot-path operations of an SD 1.5
UNet at 512 x 512 at the BASELINE configs 1-3, each at full size:
  config 1   linear 4096 x 320 -> 1280 + bias (FP16 weights)
  config 2   conv 3x3 + bias, then GroupNorm(32) + gamma + beta + SiLU, at
             [1,320,64,64], [1,640,32,32], [1,1280,8,8]
  config 3   attention 8 heads x 40, Lq 4096, Lk 4096 and 77, each + residual
Inputs are synthetic (seeded normal), weights random-init; three rotating
input sets (about 240 MB) keep every step's activations out of L2.

The JSON line follows the driver contract: value = steps/s over all GPUs,
roofline of the dominant kernel (CUDA events on its own stream), clocks
sampled during the timed region, an end-to-end number through the public API
with host buffers, the CPU baseline (the reference's single-precision forms
restated in C, oracle/ref_forms.c, on the host cores).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "stable-diffusion.assembly_b200"))

WORKLOAD = "sd15_hot_ops"
METRIC = "SD1.5 UNet hot-path op set (BASELINE configs 1-3) steps/s"
UNIT = "steps/s"


# ---------------------------------------------------------------- peaks

def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi sampled every 50 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- workload

class HotOps:
    """The op set of one step, on this rank's GPU, with per-op CUDA events."""

    SETS = 3

    def __init__(self, device, seed: int = 1234):
        import torch
        import sdb

        self.torch, self.sdb, self.dev = torch, sdb, device
        g = torch.Generator(device=device).manual_seed(seed)
        rn = lambda *s, std=1.0: torch.randn(*s, generator=g, device=device) * std
        # Weights (constant across steps; packed once by the store).
        self.w_lin = rn(1280, 320, std=0.02).half()
        self.b_lin = rn(1280, std=0.02)
        self.convs = []
        for c, hw in ((320, 64), (640, 32), (1280, 8)):
            self.convs.append(dict(c=c, hw=hw, w=rn(c, c, 3, 3, std=1 / math.sqrt(9 * c)).half(),
                                   b=rn(1, c, 1, 1, std=0.02), gamma=1 + rn(1, c, 1, 1, std=0.1),
                                   beta=rn(1, c, 1, 1, std=0.1)))
        # Rotating activation sets.
        self.sets = []
        for _ in range(self.SETS):
            s = dict(x_lin=rn(4096, 320), y_lin=torch.empty(4096, 1280, device=device))
            for i, cv in enumerate(self.convs):
                s[f"x_conv{i}"] = rn(1, cv["c"], cv["hw"], cv["hw"])
                s[f"y_conv{i}"] = torch.empty(1, cv["c"], cv["hw"], cv["hw"], device=device)
                s[f"z_conv{i}"] = torch.empty_like(s[f"y_conv{i}"])
            for lk in (4096, 77):
                s[f"q{lk}"] = rn(1, 4096, 320)
                s[f"k{lk}"] = rn(1, lk, 320)
                s[f"v{lk}"] = rn(1, lk, 320)
                s[f"r{lk}"] = rn(1, 4096, 320)
                s[f"o{lk}"] = torch.empty(1, 4096, 320, device=device)
            self.sets.append(s)
        self.ops = self._ops()

    def _ops(self):
        """(name, work, bound, fn(set)) -- work in FLOPs (tensor) or bytes (hbm), the reference's convention."""
        sdb = self.sdb
        ops = []
        ops.append(("linear_4096x320x1280_bias", 4096 * 1280 * 4 + 4096 * 320 * 4 + 1280 * 320 * 2, "hbm",
                    lambda s: sdb.mul_mat(self.w_lin, s["x_lin"], s["y_lin"], chain=sdb.Chain().add(self.b_lin))))
        for i, cv in enumerate(self.convs):
            c, hw = cv["c"], cv["hw"]
            flops = 2 * 9 * c * c * hw * hw
            ops.append((f"conv3x3_{c}x{hw}x{hw}_bias", flops, "tensor",
                        lambda s, i=i, cv=cv: sdb.conv2d(cv["w"], s[f"x_conv{i}"], (1, 1), (1, 1), (1, 1),
                                                         out=s[f"y_conv{i}"], chain=sdb.Chain().add(cv["b"]))))
            gn_bytes = 2 * c * hw * hw * 4
            ops.append((f"groupnorm32_silu_{c}x{hw}x{hw}", gn_bytes, "hbm",
                        lambda s, i=i, cv=cv: sdb.group_norm(s[f"y_conv{i}"], 32, 1e-5, out=s[f"z_conv{i}"],
                                                             chain=sdb.Chain().mul(cv["gamma"]).add(cv["beta"]).silu())))
        for lk in (4096, 77):
            flops = 4 * 40 * 8 * 4096 * lk
            ops.append((f"attention_h8d40_q4096_k{lk}_residual", flops, "tensor" if lk > 256 else "hbm",
                        lambda s, lk=lk: sdb.attention_heads(
                            s[f"q{lk}"], s[f"k{lk}"], s[f"v{lk}"], 8, 8, 40 ** -0.5, out=s[f"o{lk}"],
                            chain=sdb.Chain().add(s[f"r{lk}"], nb=[1, 40, 320, 4096 * 320]))))
        # Memory-bound attention's work is its bytes: q, k, v, residual in, out.
        name, _, bound, fn = ops[-1]
        ops[-1] = (name, (4096 * 320 * 3 + 77 * 320 * 2) * 4, bound, fn)
        return ops

    def step(self, i: int, events=None):
        s = self.sets[i % self.SETS]
        for j, (_, _, _, fn) in enumerate(self.ops):
            if events is not None:
                events[j][0].record()
            fn(s)
            if events is not None:
                events[j][1].record()

    # End to end: the same op set with its inputs coming from pinned host
    # memory and its outputs going back, every step.
    def e2e_buffers(self):
        torch = self.torch
        s = self.sets[0]
        ins = ["x_lin"] + [f"x_conv{i}" for i in range(3)] + [f"{p}{lk}" for lk in (4096, 77) for p in "qkvr"]
        outs = ["y_lin"] + [f"z_conv{i}" for i in range(3)] + ["o4096", "o77"]
        h_in = {k: s[k].cpu().pin_memory() for k in ins}
        h_out = {k: torch.empty(s[k].shape, dtype=s[k].dtype).pin_memory() for k in outs}
        return ins, outs, h_in, h_out

    def e2e_step(self, ins, outs, h_in, h_out):
        s = self.sets[0]
        for k in ins:
            s[k].copy_(h_in[k], non_blocking=True)
        for _, _, _, fn in self.ops:
            fn(s)
        for k in outs:
            h_out[k].copy_(s[k], non_blocking=True)


# ---------------------------------------------------------------- CPU baseline

def cpu_baseline(budget_s: float = 20.0) -> dict:
    """The reference's single-precision forms (oracle/ref_forms.c) on a sample of the step.

    Each op runs on a fraction of its work (rows, output channels, queries),
    its time scaled up by the inverse fraction; the step estimate is the sum.
    """
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import ref_forms

    rng = np.random.default_rng(0)
    lib_threads = ref_forms.threads()
    total = 0.0
    parts = {}

    def timed(fn):
        fn()  # warm (first-touch, thread pool)
        t0 = time.perf_counter()
        fn()
        return time.perf_counter() - t0

    # config 1: 512 of 4096 rows.
    x = rng.standard_normal((512, 320)).astype(np.float32)
    w = (rng.standard_normal((1280, 320)) * 0.02).astype(np.float16)
    t = timed(lambda: ref_forms.mul_mat(w, x)) * (4096 / 512)
    parts["linear"] = t
    for c, hw, frac in ((320, 64, 16), (640, 32, 16), (1280, 8, 8)):
        xc = rng.standard_normal((1, c, hw, hw)).astype(np.float32)
        wc = (rng.standard_normal((c, c, 3, 3)) / math.sqrt(9 * c)).astype(np.float16)
        n = c // frac
        t = timed(lambda: ref_forms.conv2d(wc, xc, (1, 1), (1, 1), (1, 1), oc_range=(0, n))) * frac
        parts[f"conv{c}"] = t
        y = rng.standard_normal((1, c, hw, hw)).astype(np.float32)
        g = np.ones(c, np.float32)
        parts[f"gn{c}"] = timed(lambda: ref_forms.group_norm(y, 32, 1e-5, g, g, True))
    for lk, qn in ((4096, 128), (77, 1024)):
        q = rng.standard_normal((1, 4096, 320)).astype(np.float32)
        k = rng.standard_normal((1, lk, 320)).astype(np.float32)
        v = rng.standard_normal((1, lk, 320)).astype(np.float32)
        t = timed(lambda: ref_forms.attention(q, k, v, 8, 8, 40 ** -0.5, q_range=(0, qn))) * (4096 / qn)
        parts[f"attention_k{lk}"] = t
    total = sum(parts.values())
    return {"value": 1.0 / total, "unit": UNIT, "cores": lib_threads, "kind": "port",
            "sample": "linear 512/4096 rows, convs 1/16 (1/8 at 1280) of output channels, attention 128 (Lk 4096) "
                      "and 1024 (Lk 77) of 4096 queries; GroupNorm whole; each timed once after a warm run, "
                      "scaled by the inverse fraction",
            "seconds_per_step": total, "parts_s": {k: round(v, 4) for k, v in parts.items()},
            "cpu": _cpu_model()}


def _cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------- main

def run_reference(args) -> None:
    """The reference arm: the reference's CPU forms (restated in C) on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    for _ in range(max(0, args.warmup)):
        pass
    samples = [cpu_baseline() for _ in range(max(1, min(3, args.steps)))]
    best = max(samples, key=lambda s: s["value"])
    line = {"metric": METRIC, "value": best["value"], "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 / best["value"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "sample": best["sample"]},
            "cpu_baseline": {k: best[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": best["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    import sdb

    sdb.load()
    work = HotOps(dev, seed=1234)
    nops = len(work.ops)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # Each step's launches are captured once per input set into a CUDA graph
    # and replayed: the device time of the kernels, without the host's
    # per-call work (that is in the end-to-end number below).  Warm-up on the
    # capture stream sizes the library's workspace before capture.
    cap = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(cap):
        for i in range(max(3, args.warmup)):
            work.step(i)
    torch.cuda.synchronize()
    graphs, op_graphs = [], [[None] * work.SETS for _ in range(nops)]
    launches_per_step = 0
    for sidx in range(work.SETS):
        g = torch.cuda.CUDAGraph()
        n0 = sdb.launch_count()
        with torch.cuda.graph(g, stream=cap):
            work.step(sidx)
        launches_per_step = sdb.launch_count() - n0
        graphs.append(g)
        for j, (_, _, _, fn) in enumerate(work.ops):
            gj = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gj, stream=cap):
                fn(work.sets[sidx])
            op_graphs[j][sidx] = gj
    torch.cuda.synchronize()
    for i in range(args.warmup):
        graphs[i % work.SETS].replay()
    torch.cuda.synchronize()

    # Timed region: K steps.
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start.record()
        for i in range(args.steps):
            graphs[i % work.SETS].replay()
        end.record()
        torch.cuda.synchronize()
    launches = launches_per_step * args.steps
    barrier()
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)

    # Each op alone (graph replays over the rotating sets), for the roofline.
    per_op_ms = []
    reps = max(30, min(300, args.steps))
    for j in range(nops):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            op_graphs[j][i % work.SETS].replay()
        e1.record()
        torch.cuda.synchronize()
        per_op_ms.append(e0.elapsed_time(e1) / reps)
    del graphs, op_graphs

    # End to end through the public API with host buffers.
    ins, outs, h_in, h_out = work.e2e_buffers()
    for _ in range(2):
        work.e2e_step(ins, outs, h_in, h_out)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        work.e2e_step(ins, outs, h_in, h_out)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    h2d = sum(h_in[k].numel() * h_in[k].element_size() for k in ins)
    d2h = sum(h_out[k].numel() * h_out[k].element_size() for k in outs)

    status = sdb.device_status(clear=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks = measured_peaks()
    dom = max(range(nops), key=lambda j: per_op_ms[j])
    name, work_units, bound, _ = work.ops[dom]
    dur_s = per_op_ms[dom] * 1e-3
    if bound == "tensor":
        achieved = work_units / dur_s / 1e12
        peak, unit = peaks["bf16_tflops"], "TFLOP/s"
    else:
        achieved = work_units / dur_s / 1e9
        peak, unit = peaks["hbm_gbs"], "GB/s"
    traffic = None
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get(name)
    line = {
        "metric": METRIC, "value": world * 1e3 / ms, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "ops": [o[0] for o in work.ops], "parallelism": f"replicas x{world}",
                   "l2": "3 rotating input sets (~240 MB) > L2", "weights": "random-init FP16, packed once",
                   "timing": "CUDA-graph replay of each step's launches; per-op times from graphs of each op"},
        "roofline": {"kernel": name, "bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak, "peak_source": peaks["source"], "traffic": traffic,
                     "work_per_launch": work_units, "avg_launch_ms": per_op_ms[dom]},
        "per_op_ms": {work.ops[j][0]: round(per_op_ms[j], 5) for j in range(nops)},
        "e2e": {"value": world * 1e3 / e2e_ms, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "device_status": status,
    }
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline()
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        line["cpu_baseline"]["cpu"] = cb["cpu"]
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
