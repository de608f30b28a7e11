#!/usr/bin/env python
"""Benchmark of the B200 kernels behind stable-diffusion.assembly's hook surface.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload unet|hot_ops]

One process per GPU (torchrun for N > 1).  The default workload shards a fixed
8-image batch by image over the N GPUs (strong scaling, no data-path
collective); the step time is the max over ranks, and rank 0 prints one JSON
line.

Workload "sd15_unet_step" (default; benchmark config 4): one sampler step of SD
1.5 at 512 x 512 -- the UNet forward on the classifier-free-guidance batch of 2
(latent 64 x 64, context 2 x 77 x 768; ~860M random-init FP16 weights) and the
fused guidance (scale 7) + Euler update -- captured once as a CUDA graph and
replayed K times; ms_per_step is the UNet ms/step, value the whole job's UNet
steps/s.  A second, eager pass with CUDA events around every library call
gives the step's per-class times and the roofline of the dominant class.
Weights (1.7 GB) and activations exceed L2 every step.

Workload "sd15_hot_ops" (--workload hot_ops): the benchmark configs 1-3 op set.

The JSON line follows the driver contract: roofline of the dominant kernel
class, clocks sampled during the timed region, an end-to-end number through
the public API with host buffers (the latent and context in, the latent out,
every step), and the CPU baseline: the reference's single-precision forms
restated in C (oracle/ref_forms.c) on the host cores, on a sample of the
step's operations.
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

HOT_WORKLOAD = "sd15_hot_ops"
HOT_METRIC = "SD1.5 UNet hot-path op set (benchmark configs 1-3) steps/s"
HOT_UNIT = "steps/s"
UNET_WORKLOAD = "sd15_unet_step"
UNET_METRIC = ("UNet ms/step + VAE ms (SD1.5 512x512, CFG 7, Euler; the 8-image batch over the GPUs): whole-job "
               "image-steps/s (an image-step: one image's UNet step on its CFG batch of 2); ms_per_step is the "
               "job's UNet step")
UNET_UNIT = "image-steps/s"
SAMPLER_STEPS = 20
IMAGES = 8        # benchmark config 4: batches of 8 images, sharded by image over 1/2/4/8 GPUs


# ---------------------------------------------------------------- peaks

def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


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
        """(name, work, bound, fn(set)) -- benchmark configs 1-3, work in FLOPs (tensor) or the least bytes
        moved (hbm), by the reference's convention (bench.cc:82-124, profile.cc:65-81)."""
        sdb = self.sdb
        ops = []
        ops.append(("config1_linear_4096x320x1280_bias", 4096 * 1280 * 4 + 4096 * 320 * 4 + 1280 * 320 * 2 + 1280 * 4,
                    "hbm",
                    lambda s: sdb.mul_mat(self.w_lin, s["x_lin"], s["y_lin"], chain=sdb.Chain().add(self.b_lin))))
        for i, (tag, cv) in enumerate(zip("abc", self.convs)):
            c, hw = cv["c"], cv["hw"]
            flops = 2 * 9 * c * c * hw * hw
            # 8x8: the weights' bytes bound it (about 63 FLOP a byte at 1280 channels).
            work, bound = (flops, "tensor") if hw > 8 else (c * c * 9 * 2 + 2 * c * hw * hw * 4, "hbm")

            def conv_gn(s, i=i, cv=cv):
                sdb.conv2d(cv["w"], s[f"x_conv{i}"], (1, 1), (1, 1), (1, 1), out=s[f"y_conv{i}"],
                           chain=sdb.Chain().add(cv["b"]))
                sdb.group_norm(s[f"y_conv{i}"], 32, 1e-5, out=s[f"z_conv{i}"],
                               chain=sdb.Chain().mul(cv["gamma"]).add(cv["beta"]).silu())

            ops.append((f"config2{tag}_conv3x3_{c}x{hw}x{hw}_bias_gn32_silu", work, bound, conv_gn))
        for tag, lk in (("a", 4096), ("b", 77)):
            flops = 4 * 40 * 8 * 4096 * lk
            for residual in (False, True):
                if lk > 256:
                    work, bound = flops, "tensor"
                else:   # cross-attention: q, k, v (and the residual) in, the output out
                    work, bound = (4096 * 320 * (3 if residual else 2) + 2 * 77 * 320) * 4, "hbm"

                def attn(s, lk=lk, residual=residual):
                    ch = sdb.Chain().add(s[f"r{lk}"], nb=[1, 40, 320, 4096 * 320]) if residual else None
                    sdb.attention_heads(s[f"q{lk}"], s[f"k{lk}"], s[f"v{lk}"], 8, 8, 40 ** -0.5, out=s[f"o{lk}"],
                                        chain=ch)

                kind = "self" if lk > 256 else "cross"
                ops.append((f"config3{tag}_{kind}_attention_h8d40_q4096_k{lk}" + ("_residual" if residual else ""),
                            work, bound, attn))
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
    return {"value": 1.0 / total, "unit": HOT_UNIT, "cores": lib_threads, "kind": "port",
            "sample": "linear 512/4096 rows, convs 1/16 (1/8 at 1280) of output channels, attention 128 (Lk 4096) "
                      "and 1024 (Lk 77) of 4096 queries; GroupNorm whole; each timed once after a warm run, "
                      "scaled by the inverse fraction",
            "seconds_per_step": total, "parts_s": {k: round(v, 4) for k, v in parts.items()},
            "cpu": _cpu_model()}


def unet_ops(batch: int = 2, h: int = 64, w: int = 64, ctx: int = 77) -> list[tuple]:
    """The operations of one SD 1.5 UNet forward, in order, with their shapes -- the calls
    stable-diffusion.assembly_b200/unet.py makes:
      ("conv", N, IC, OC, H, W, K, stride)   ("linear", M, K, N)   ("geglu", M, K, 2 x out)
      ("attn", B, heads, Lq, Lk, d)          ("gn", N, C, H, W)     ("ln", M, C)
      ("cat", N, C1, C2, H, W)               ("upsample", N, C, H, W) (nearest, 2x)"""
    import unet as U

    c = U.SD15
    mc, td = c.model_channels, c.model_channels * c.time_dim_mult
    ops: list[tuple] = []
    blocks: list[tuple] = []   # ("res", cin, cout, hh, ww) / ("tr", ch, hh, ww) / ("down"|"up", ...) / ("cat", ...)
    chans, ch, hh, ww = [mc], mc, h, w
    for lvl, mult in enumerate(c.channel_mult):
        for _ in range(c.num_res_blocks):
            blocks.append(("res", ch, mult * mc, hh, ww))
            ch = mult * mc
            if lvl in c.attention_levels:
                blocks.append(("tr", ch, hh, ww))
            chans.append(ch)
        if lvl != len(c.channel_mult) - 1:
            blocks.append(("down", ch, hh, ww))
            hh, ww = (hh + 1) // 2, (ww + 1) // 2
            chans.append(ch)
    blocks += [("res", ch, ch, hh, ww), ("tr", ch, hh, ww), ("res", ch, ch, hh, ww)]
    for lvl, mult in reversed(list(enumerate(c.channel_mult))):
        for _ in range(c.num_res_blocks + 1):
            skip = chans.pop()
            blocks.append(("cat", ch, skip, hh, ww))
            blocks.append(("res", ch + skip, mult * mc, hh, ww))
            ch = mult * mc
            if lvl in c.attention_levels:
                blocks.append(("tr", ch, hh, ww))
        if lvl != 0:
            blocks.append(("up", ch, hh, ww))
            hh, ww = hh * 2, ww * 2
    emb_total = sum(b[2] for b in blocks if b[0] == "res")
    kv_total = sum(2 * b[1] for b in blocks if b[0] == "tr")
    ops += [("linear", batch, mc, td), ("linear", batch, td, td), ("linear", batch, td, emb_total),
            ("linear", batch * ctx, c.context_dim, kv_total), ("conv", batch, c.in_channels, mc, h, w, 3, 1)]
    for b in blocks:
        if b[0] == "res":
            _, cin, cout, bh, bw = b
            ops += [("gn", batch, cin, bh, bw), ("conv", batch, cin, cout, bh, bw, 3, 1), ("gn", batch, cout, bh, bw)]
            if cin != cout:
                ops.append(("conv", batch, cin, cout, bh, bw, 1, 1))
            ops.append(("conv", batch, cout, cout, bh, bw, 3, 1))
        elif b[0] == "tr":
            _, cc, bh, bw = b
            m = batch * bh * bw
            ops += [("gn", batch, cc, bh, bw), ("linear", m, cc, cc),
                    ("ln", m, cc), ("linear", m, cc, 3 * cc), ("attn", batch, c.heads, bh * bw, bh * bw, cc // c.heads),
                    ("linear", m, cc, cc),
                    ("ln", m, cc), ("linear", m, cc, cc), ("attn", batch, c.heads, bh * bw, ctx, cc // c.heads),
                    ("linear", m, cc, cc),
                    ("ln", m, cc), ("geglu", m, cc, 8 * cc), ("linear", m, 4 * cc, cc), ("linear", m, cc, cc)]
        elif b[0] == "down":
            _, cc, bh, bw = b
            ops.append(("conv", batch, cc, cc, bh, bw, 3, 2))
        elif b[0] == "up":
            _, cc, bh, bw = b
            ops += [("upsample", batch, cc, bh, bw), ("conv", batch, cc, cc, 2 * bh, 2 * bw, 3, 1)]
        elif b[0] == "cat":
            _, c1, c2, bh, bw = b
            ops.append(("cat", batch, c1, c2, bh, bw))
    ops += [("gn", batch, mc, h, w), ("conv", batch, mc, c.out_channels, h, w, 3, 1)]
    return ops


def _reference_kernels():
    """oracle/_ref/libsdasm_ref.so -- the reference's own x86-64 micro-kernels assembled from its sources
    (oracle/ref_asm.py) with this project's threaded driver -- when it was built, else None."""
    import ctypes

    lib_path = ROOT / "oracle" / "_ref" / "libsdasm_ref.so"
    if not lib_path.exists():
        return None
    try:
        lib = ctypes.CDLL(str(lib_path))
    except OSError:
        return None
    P, i = ctypes.c_void_p, ctypes.c_int
    lib.refk_mul_mat_mt.argtypes = [P, i, i, P, i, P]
    lib.refk_conv2d_mt.argtypes = [P, i, i, i, i, P, i, i, i, i, i, i, i, P]
    lib.refk_winograd_mt.argtypes = [P, i, i, P, i, i, i, i, i, P]
    lib.refk_attention_mt.argtypes = [P, P, P, P, i, i, i, i, i, i, ctypes.c_float, i]
    lib.refk_gated_gelu.argtypes = [P, P, P, ctypes.c_int64]
    lib.refk_set_threads.argtypes = [i]
    return lib


def host_threads() -> int:
    """The host cores this process may run on (a launcher's OMP_NUM_THREADS does not count)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def winograd_form(n: int, oh: int, ow: int) -> int:
    """The reference's choice for a 3x3 stride-1 convolution (winograd.cc:194-196, 1204-1206, 2107-2123,
    default Tuning): Winograd from 1024 outputs an image, or when all images have at most 256 F(2x2)
    tiles; F(4x4) from 256 outputs an image (FP16 weights), else F(2x2); 0: direct."""
    small = n * ((ow + 1) // 2) * ((oh + 1) // 2) <= 256
    if not (ow * oh >= 1024 or small):
        return 0
    return 4 if ow * oh >= 256 else 2


class CpuUNetStep:
    """One image's SD 1.5 UNet step (its CFG batch of 2) on the reference's CPU path, every operation whole.

    Products -- linear layers, GEGLU, direct convolutions, attention's two products, Winograd's
    (F+2)^2 products -- run the reference's own micro-kernels (assembled from its sources:
    sdasm_gemm_6x32_avx512 / 6x16_avx512 on AVX-512 hosts, else sdasm_gemm_6x16_avx2) as its
    mul_mat / conv2d / attention drive them, 3x3 convolutions in the form the reference picks
    (Winograd F(4x4) or F(2x2) by its thresholds, transforms restated in C); GEGLU's gate by its
    sdasm_gated_gelu_avx2; GroupNorm, LayerNorm and attention's softmax in its single-precision
    forms restated in C; the concatenations and upsamplings as copies.  Every operation of the
    step runs once per call, on all host cores; weights are distinct per layer (the UNet's 859.5M
    FP16 numbers), their widened panels kept between calls as the reference's store keeps them.
    """

    def __init__(self):
        import ctypes

        import numpy as np

        sys.path.insert(0, str(ROOT / "oracle"))
        import ref_forms

        self.np, self.ctypes, self.rf = np, ctypes, ref_forms
        self.refk = _reference_kernels()
        if self.refk is None:
            raise RuntimeError("oracle/_ref/libsdasm_ref.so is not built")
        self.cores = host_threads()
        self.refk.refk_set_threads(self.cores)
        ref_forms.set_threads(self.cores)
        rng = np.random.default_rng(0)
        self.ops = unet_ops()
        # Weights: one FP16 pool, each layer its own slice (distinct addresses, as the model's).
        sizes = []
        for op in self.ops:
            if op[0] == "conv":
                _, b, ic, oc, hh, ww, k, st = op
                sizes.append(oc * ic * k * k)
            elif op[0] in ("linear", "geglu"):
                sizes.append(op[2] * op[3])
            else:
                sizes.append(0)
        block = (rng.standard_normal(1 << 22) * 0.05).astype(np.float16)
        total = sum(sizes)
        self.pool = np.empty(total + 64, np.float16)
        for o in range(0, total, block.size):
            n = min(block.size, total - o)
            self.pool[o:o + n] = block[:n]
        self.weights, off = [], 0
        for n in sizes:
            self.weights.append(self.pool[off:off + n] if n else None)
            off += (n + 31) // 32 * 32 if n else 0
        # Activations: inputs and outputs per distinct shape (reused across occurrences).
        self.bufs: dict = {}

    def _buf(self, key, shape):
        np = self.np
        if key not in self.bufs:
            self.bufs[key] = (np.random.default_rng(len(self.bufs)).standard_normal(shape) * 0.5).astype(np.float32)
        return self.bufs[key]

    def run(self) -> dict:
        """Runs every operation once; returns seconds per kind."""
        np, P = self.np, self.ctypes.c_void_p
        ptr = lambda a: a.ctypes.data_as(P)
        refk, rf = self.refk, self.rf
        parts: dict[str, float] = {}
        for op, wt in zip(self.ops, self.weights):
            kind = op[0]
            t0 = time.perf_counter()
            if kind == "conv":
                _, b, ic, oc, hh, ww, k, st = op
                x = self._buf(("x", b, ic, hh, ww), (b, ic, hh, ww))
                oh, ow = (hh + 2 * (k // 2) - k) // st + 1, (ww + 2 * (k // 2) - k) // st + 1
                y = self._buf(("y", b, oh, ow, oc), (b, oh, ow, oc))
                f = winograd_form(b, oh, ow) if (k == 3 and st == 1) else 0
                if f:
                    refk.refk_winograd_mt(ptr(wt), oc, ic, ptr(x), b, hh, ww, 1, f, ptr(y))
                    kind = f"conv3x3_winograd_f{f}"
                else:
                    refk.refk_conv2d_mt(ptr(wt), oc, ic, k, k, ptr(x), b, hh, ww, st, k // 2, oh, ow, ptr(y))
                    kind = f"conv{k}x{k}_direct"
            elif kind in ("linear", "geglu"):
                _, m, kk, nn = op
                x = self._buf(("x", m, kk), (m, kk))
                y = self._buf(("y", m, nn), (m, nn))
                refk.refk_mul_mat_mt(ptr(wt), nn, kk, ptr(x), m, ptr(y))
                if kind == "geglu":
                    half = nn // 2
                    out = self._buf(("g", m, half), (m, half))
                    xs, gs = np.ascontiguousarray(y[:, :half]), np.ascontiguousarray(y[:, half:])
                    refk.refk_gated_gelu(ptr(out), ptr(xs), ptr(gs), out.size)
            elif kind == "attn":
                _, b, heads, lq, lk, d = op
                q = self._buf(("q", b, lq, heads * d), (b, lq, heads * d))
                kv = self._buf(("kv", b, lk, heads * d), (b, lk, heads * d))
                o = self._buf(("o", b, lq, heads * d), (b, lq, heads * d))
                refk.refk_attention_mt(ptr(q), ptr(kv), ptr(kv), ptr(o), b, heads, lq, lk, d, d, d ** -0.5, lq)
                kind = "self_attention" if lq == lk else "cross_attention"
            elif kind == "gn":
                _, b, cc, hh, ww = op
                x = self._buf(("x", b, cc, hh, ww), (b, cc, hh, ww))
                g = self._buf(("gamma", cc), (cc,))
                rf.group_norm(x, 32, 1e-5, g, g, True)
            elif kind == "ln":
                _, m, cc = op
                x = self._buf(("x", m, cc), (m, cc))
                g = self._buf(("gamma", cc), (cc,))
                rf.norm(x, 1e-5, g, g, out=self._buf(("ln", m, cc), (m, cc)))
            elif kind == "cat":
                _, b, c1, c2, hh, ww = op
                a = self._buf(("x", b, c1, hh, ww), (b, c1, hh, ww))
                bb = self._buf(("x", b, c2, hh, ww), (b, c2, hh, ww))
                out = self._buf(("x", b, c1 + c2, hh, ww), (b, c1 + c2, hh, ww))
                out[:, :c1] = a
                out[:, c1:] = bb
            elif kind == "upsample":
                _, b, cc, hh, ww = op
                x = self._buf(("x", b, cc, hh, ww), (b, cc, hh, ww))
                out = self._buf(("x", b, cc, 2 * hh, 2 * ww), (b, cc, 2 * hh, 2 * ww))
                out.reshape(b, cc, hh, 2, ww, 2)[...] = x[:, :, :, None, :, None]
            parts[kind] = parts.get(kind, 0.0) + time.perf_counter() - t0
        return parts

    def describe(self) -> str:
        isa = "AVX-512 (sdasm_gemm_6x32_avx512)" if self.refk.refk_isa() else "AVX2 (sdasm_gemm_6x16_avx2)"
        return ("one image's SD 1.5 UNet step (CFG batch 2, 64x64 latent) per step, every operation whole: products "
                f"on the reference's own {isa} micro-kernel assembled from its sources, 3x3 convolutions by "
                "Winograd F(4x4)/F(2x2) where the reference takes them (transforms restated in C), GEGLU's gate "
                "by its sdasm_gated_gelu_avx2, GroupNorm/LayerNorm/softmax in its single-precision forms restated "
                f"in C, concatenations and upsamplings as copies; {self.cores} host threads")


_CPU_STEP = None


def cpu_unet_step(steps: int = 1) -> dict:
    """The reference's CPU path timed on `steps` whole image-steps after one untimed (the fastest counts,
    as tools/bench.cc:431-451 takes the fastest of its runs)."""
    global _CPU_STEP
    if _CPU_STEP is None:
        _CPU_STEP = CpuUNetStep()
    cs = _CPU_STEP
    cs.run()
    best, best_parts = None, None
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        parts = cs.run()
        dt = time.perf_counter() - t0
        if best is None or dt < best:
            best, best_parts = dt, parts
    return {"value": 1.0 / best, "unit": UNET_UNIT, "cores": cs.cores, "kind": "reference",
            "sample": cs.describe(), "seconds_per_step": best,
            "parts_s": {k: round(v, 3) for k, v in sorted(best_parts.items(), key=lambda kv: -kv[1])},
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

def unet_config(world: int, tune: str | None) -> dict:
    """The sd15_unet_step workload's description, the same for both arms."""
    per = max(1, IMAGES // world)
    return {"workload": UNET_WORKLOAD, "resolution": "512x512 (latent 64x64)",
            "images": f"{IMAGES}-image batch, {per} a GPU",
            "batch": f"{2 * per} a GPU ({per} image(s) x CFG 2)",
            "tuning": tune or "default (FP32-accurate products)",
            "context": "2x77x768", "sampler": f"Euler, {SAMPLER_STEPS} steps, CFG 7",
            "weights": "random-init FP16, the SD 1.5 UNet's 859.5M parameters, packed once",
            "parallelism": f"images over {world} GPU(s): {per} a GPU, no data-path collective",
            "l2": "weights (1.7 GB) and activations exceed L2 every step",
            "timing": "CUDA-graph replay of the UNet forward + the guidance/Euler kernel per step",
            "vae": "SD 1.5 decoder, a GPU's 64x64 latents to 512x512 images, random-init FP16 weights "
                   "(49.5M parameters); vae_ms is one decode of them, a CUDA-graph replay; imgs_per_s "
                   f"counts {SAMPLER_STEPS} UNet steps and the decode"}


def run_reference(args) -> None:
    """The reference arm: the reference's CPU path on the host cores, on this arm's workload and metric.

    UNet workload: W untimed and K timed steps, each one image's whole UNet step (its CFG batch of 2)
    through CpuUNetStep -- every operation of the step run in full, nothing scaled up; value = the K
    image-steps over their measured seconds.  Under torchrun rank 0 alone runs it, on all the cores
    its affinity allows."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    unet = args.workload == "unet"
    if not unet:
        best = max((cpu_baseline() for _ in range(max(1, min(3, args.steps)))), key=lambda s: s["value"])
        line = {"metric": HOT_METRIC, "value": best["value"], "unit": HOT_UNIT, "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / best["value"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "impl": "reference", "config": {"workload": HOT_WORKLOAD},
                "cpu_baseline": {k: best[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": best["value"], "unit": HOT_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    global _CPU_STEP
    _CPU_STEP = _CPU_STEP or CpuUNetStep()
    cs = _CPU_STEP
    for _ in range(args.warmup):
        cs.run()
    parts: dict[str, float] = {}
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for k, v in cs.run().items():
            parts[k] = parts.get(k, 0.0) + v
    seconds = time.perf_counter() - t0
    value = args.steps / seconds
    line = {"metric": UNET_METRIC, "value": value, "unit": UNET_UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * seconds / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": unet_config(args.gpus, args.tune),
            "sample": cs.describe(),
            "cpu_baseline": {"value": value, "unit": UNET_UNIT, "cores": cs.cores, "kind": "reference",
                             "sample": cs.describe(), "cpu": _cpu_model(),
                             "parts_s_per_step": {k: round(v / args.steps, 3)
                                                  for k, v in sorted(parts.items(), key=lambda kv: -kv[1])}},
            "e2e": {"value": value, "unit": UNET_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def hot_op_configs(torch, dev, reps: int = 30) -> dict:
    """benchmark configs 1-3 timed op by op on this GPU (CUDA-graph replays over three rotating input
    sets larger than L2), each against its roofline: tensor-bound ops by the reference's FLOP count over
    the measured bf16 burst peak, memory-bound ones by their least bytes over the measured HBM copy rate
    (MEASURED_PEAKS.json)."""
    work = HotOps(dev, seed=1234)
    cap = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(cap):
        for i in range(3):
            work.step(i)
    torch.cuda.synchronize()
    graphs = []
    for _, _, _, fn in work.ops:
        gs = []
        for sidx in range(work.SETS):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                fn(work.sets[sidx])
            gs.append(g)
        graphs.append(gs)
    torch.cuda.synchronize()
    peaks = measured_peaks()
    profiles = {p.stem: str(p.relative_to(ROOT)) for p in (ROOT / "profiles").glob("*.md")}
    out = {}
    for (name, units, bound, _), gs in zip(work.ops, graphs):
        for i in range(3):
            gs[i % work.SETS].replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            gs[i % work.SETS].replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        if bound == "tensor":
            achieved, peak, unit = units / (ms * 1e-3) / 1e12, peaks["bf16_tflops"], "TFLOP/s"
        else:
            achieved, peak, unit = units / (ms * 1e-3) / 1e9, peaks["hbm_gbs"], "GB/s"
        key = name.split("_", 1)[0]
        prof = [v for k, v in profiles.items() if k.startswith(key)]
        out[name] = {"ms": round(ms, 5), "bound": bound, "work": units, "achieved": round(achieved, 1),
                     "peak": peak, "unit": unit, "frac": round(achieved / peak, 4),
                     "peak_source": peaks["source"] + " (burst)" if bound == "tensor" else peaks["source"],
                     "profile": prof[0] if prof else None}
    del graphs
    torch.cuda.synchronize()
    return out


def run_hot_ops(args, torch, dev, dist, world, rank, local, barrier, max_over_ranks) -> None:
    import sdb

    work = HotOps(dev, seed=1234)
    nops = len(work.ops)

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
        "metric": HOT_METRIC, "value": world * 1e3 / ms, "unit": HOT_UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": HOT_WORKLOAD, "ops": [o[0] for o in work.ops], "parallelism": f"replicas x{world}",
                   "l2": "3 rotating input sets (~240 MB) > L2", "weights": "random-init FP16, packed once",
                   "timing": "CUDA-graph replay of each step's launches; per-op times from graphs of each op"},
        "roofline": {"kernel": name, "bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak, "peak_source": peaks["source"], "traffic": traffic,
                     "work_per_launch": work_units, "avg_launch_ms": per_op_ms[dom]},
        "per_op_ms": {work.ops[j][0]: round(per_op_ms[j], 5) for j in range(nops)},
        "e2e": {"value": world * 1e3 / e2e_ms, "unit": HOT_UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "device_status": status,
    }
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline()
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        line["cpu_baseline"]["cpu"] = cb["cpu"]
    print(json.dumps(line), flush=True)



# ---------------------------------------------------------------- the UNet step

CLASSES = {"conv3x3": "tensor", "conv3x3_s2": "tensor", "conv1x1": "tensor", "linear": "tensor", "geglu": "tensor",
           "self_attention": "tensor", "cross_attention": "tensor", "groupnorm": "hbm", "layernorm": "hbm",
           "glue": "hbm"}


class OpClock:
    """Records the library calls one UNet forward makes, then times each alone: the call captured
    into a CUDA graph of its own and replayed, with CUDA events on the capture stream around the
    replays (device time only).  Each call has its class and algorithmic work (FLOPs in the
    reference's convention for products, bytes read + written for the rest)."""

    NAMES = ("conv2d_nhwc", "conv2d_nhwc_normed", "mul_mat", "mul_mat_normed", "mul_mat_gated", "attention_heads",
             "group_norm_nhwc", "group_norm_stats", "norm", "mul_mat_layer_normed", "concat_channels_nhwc",
             "upscale_nearest_nhwc", "timestep_embedding")

    def __init__(self, sdb, torch):
        self.sdb, self.torch = sdb, torch
        self.records: list[tuple] = []
        self.saved = {}

    @staticmethod
    def work(name, args, out):
        if name in ("conv2d_nhwc", "conv2d_nhwc_normed"):
            w = args[0]
            oc, ic, kh, kw = w.shape
            n, oh, ow, _ = out.shape
            stride = args[3 if name == "conv2d_nhwc_normed" else 2] if len(args) > (3 if name == "conv2d_nhwc_normed"
                                                                                    else 2) else (1, 1)
            cls = "conv1x1" if kh == 1 else ("conv3x3_s2" if stride[0] == 2 else "conv3x3")
            return cls, 2 * kh * kw * ic * oc * oh * ow * n
        if name == "group_norm_stats":
            return "groupnorm", 4 * args[0].numel()
        if name == "mul_mat_layer_normed":
            w, x = args[0], args[1]
            k = w.shape[1]
            return ("geglu" if out.shape[-1] * 2 == w.shape[0] else "linear"), 2 * (x.numel() // k) * w.shape[0] * k
        if name in ("mul_mat", "mul_mat_gated", "mul_mat_normed"):
            w, x = args[0], args[1]
            k = w.shape[1]
            m = x.numel() // k
            return ("geglu" if name == "mul_mat_gated" else "linear"), 2 * m * w.shape[0] * k
        if name == "attention_heads":
            q, k, heads = args[0], args[1], args[3]
            b, lq, hd = q.shape
            lk = k.shape[1]
            return ("self_attention" if lk == lq else "cross_attention"), 4 * (hd // heads) * heads * lq * lk * b
        if name in ("group_norm_nhwc", "norm"):
            return ("groupnorm" if name == "group_norm_nhwc" else "layernorm"), 8 * args[0].numel()
        return "glue", 8 * out.numel()

    def __enter__(self):
        for name in self.NAMES:
            fn = getattr(self.sdb, name)
            self.saved[name] = fn

            def wrapped(*a, _fn=fn, _name=name, **kw):
                out = _fn(*a, **kw)
                self.records.append((_name, _fn, a, kw, out))
                return out

            setattr(self.sdb, name, wrapped)
        return self

    def __exit__(self, *exc):
        for name, fn in self.saved.items():
            setattr(self.sdb, name, fn)

    @staticmethod
    def shape_key(name, args, out) -> str:
        if name in ("conv2d_nhwc", "conv2d_nhwc_normed"):
            w, x = args[0], args[1]
            return f"conv {w.shape[1]}->{w.shape[0]} k{w.shape[2]} @{x.shape[1]}x{x.shape[2]}x{x.shape[0]}"
        if name in ("mul_mat", "mul_mat_gated", "mul_mat_normed", "mul_mat_layer_normed"):
            w, x = args[0], args[1]
            gated = name == "mul_mat_gated" or (name == "mul_mat_layer_normed" and out.shape[-1] * 2 == w.shape[0])
            return f"{'geglu' if gated else 'linear'} M{x.numel() // w.shape[1]} K{w.shape[1]} N{w.shape[0]}"
        if name == "attention_heads":
            q, k, heads = args[0], args[1], args[3]
            return f"attention L{q.shape[1]}x{k.shape[1]} d{q.shape[2] // heads} b{q.shape[0]}"
        return f"{name} {tuple(args[0].shape)}"

    def measure(self, stream, reps: int = 3) -> dict:
        torch = self.torch
        classes: dict[str, list] = {}
        self.shapes: dict[str, list] = {}
        for name, fn, a, kw, out in self.records:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                fn(*a, **kw)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                g.replay()
                e0.record()
                for _ in range(reps):
                    g.replay()
                e1.record()
            torch.cuda.synchronize()
            cls, work = self.work(name, a, out)
            c = classes.setdefault(cls, [0, 0.0, 0])
            ms = e0.elapsed_time(e1) / reps
            c[0] += work
            c[1] += ms
            c[2] += 1
            sh = self.shapes.setdefault(self.shape_key(name, a, out), [0, 0.0, 0])
            sh[0] += work
            sh[1] += ms
            sh[2] += 1
            del g
        return {k: {"work": v[0], "ms": v[1], "calls": v[2]} for k, v in classes.items()}


def measure_vae(torch, dev, latent, barrier, max_over_ranks, reps: int = 5, config=None) -> tuple[float, int]:
    """ms of one VAE decode of the latents (N, h, w, 4) (SD 1.5's decoder by default: 64 x 64 latents to
    512 x 512), a CUDA-graph replay timed with CUDA events on its stream (max over ranks), and its
    algorithmic FLOPs."""
    import vae as V

    dec = V.VAEDecoder(config or V.SD15_VAE, device=dev)
    z = latent.clone()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            dec.decode(z)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        dec.decode(z)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        graph.replay()
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        start.record(s)
        for _ in range(reps):
            graph.replay()
        end.record(s)
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end) / reps)
    flops = dec.flops(z.shape[0], z.shape[1], z.shape[2])
    del graph, dec
    return ms, flops


def measure_sdxl(torch, dev, barrier, max_over_ranks, reps: int = 5) -> dict:
    """One SDXL sampler step at 832 x 1216 (latent 152 x 104, benchmark config 5): the UNet forward on the
    classifier-free-guidance batch of 2 (context 2 x 77 x 2048, pooled text + size/crop conditioning
    2 x 2816, 2.57B random-init FP16 weights) and the guidance (scale 6) + ancestral Euler update (each
    step's fresh noise drawn before the timing), captured once and replayed; ms a step as the max over
    ranks.  Then the SDXL VAE decode of the latent to 832 x 1216."""
    import sdb
    import unet as U

    net = U.UNet(U.SDXL, device=dev, seed=20261013)
    g = torch.Generator(device=dev).manual_seed(77)
    x_in = torch.randn(2, 152, 104, 4, device=dev, generator=g)
    x = x_in[:1].clone()
    t = torch.full((2,), 700.0, device=dev)
    ctx = torch.randn(2, 77, 2048, device=dev, generator=g)
    y = torch.randn(2, 2816, device=dev, generator=g)
    out = {}

    def forward():
        out["eps"] = net.forward(x_in, t, ctx, y=y)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            forward()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        forward()
    torch.cuda.synchronize()

    noise = torch.randn(reps + 1, 152, 104, 4, device=dev, generator=g)

    def step(k):
        graph.replay()
        sdb.euler_ancestral_cfg_step(out["eps"], x, x_in, noise[k], 6.0, 1.0, 0.9, 0.7, stream=s)

    with torch.cuda.stream(s):
        step(reps)
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        start.record(s)
        for k in range(reps):
            step(k)
        end.record(s)
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end) / reps)
    flops = net.flops(2, 152, 104)
    res = {"ms_per_step": ms, "step_tflop": flops / 1e12, "tflops": flops / (ms * 1e-3) / 1e12,
           "resolution": "832x1216 (latent 152x104)", "batch": "2 (CFG 6)", "params": net.params,
           "context": "2x77x2048 + pooled/size conditioning 2x2816",
           "timing": "CUDA-graph replay of the UNet forward + the guidance/ancestral-Euler kernel per step"}
    del graph, net
    torch.cuda.empty_cache()
    import vae as V

    vae_ms, vae_flops = measure_vae(torch, dev, x.clone(), barrier, max_over_ranks, reps=3, config=V.SDXL_VAE)
    res.update({"vae_ms": vae_ms, "vae_tflops": vae_flops / (vae_ms * 1e-3) / 1e12,
                "imgs_per_s": 1000.0 / (20 * ms + vae_ms),
                "vae": "SDXL decoder (SD's first-stage decoder, latents scaled by 0.13025), 152x104 latent to "
                       "1216x832, random-init FP16 weights; imgs_per_s counts 20 steps and one decode"})
    torch.cuda.empty_cache()
    return res


def run_cfg_split(args, torch, dev, dist, world, rank, local, barrier, max_over_ranks) -> None:
    """SD 1.5 with classifier-free guidance split over GPU pairs (--cfg-split): each rank runs the UNet on one
    half of the guidance batch (batch 1), the pair all-gathers its eps each step (NCCL), both take the same
    update.  value = images a step x steps/s over the job (world / 2 images).  Each rank's work is one
    guidance half whatever N, and the job's images grow with N: weak scaling (the mode for one image's
    latency; the default image sharding is the strong-scaling throughput mode)."""
    import sdb
    import unet as U

    if world % 2:
        raise SystemExit("--cfg-split needs an even number of ranks")
    groups = U.pair_groups(dist, world)
    net = U.UNet(U.SD15, device=dev, seed=20261011)
    sampler = U.PairSampler(net, dist, groups[rank // 2], rank % 2, 64, 64, steps=SAMPLER_STEPS)
    g = torch.Generator(device=dev).manual_seed(1234 + rank // 2)
    latent = torch.randn(1, 64, 64, 4, device=dev, generator=g)
    context = torch.randn(2, 77, 768, device=dev, generator=g)
    sampler.x.copy_(latent * sampler.sigmas[0])
    sampler.context.copy_(context[rank % 2:rank % 2 + 1])
    sampler.set_step(0)
    sampler.capture(warmup=max(3, args.warmup))
    for i in range(args.warmup):
        sampler.step(i % SAMPLER_STEPS)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(sampler.stream)
        for i in range(args.steps):
            sampler.step(i % SAMPLER_STEPS)
        end.record(sampler.stream)
        torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    # Both ranks of a pair hold the same latent after every step.
    both = torch.empty(2, *sampler.x.shape[1:], device=dev)
    U.gather_guidance(dist, groups[rank // 2], sampler.x, both)
    same = torch.tensor([1.0 if torch.equal(both[0], both[1]) else 0.0], device=dev)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    status = sdb.device_status(clear=True)
    del sampler
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": UNET_METRIC, "value": (world // 2) * 1e3 / ms, "unit": UNET_UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": UNET_WORKLOAD + "_cfg_split", "resolution": "512x512 (latent 64x64)",
                   "batch": "1 a rank (one guidance half), 2 a pair",
                   "parallelism": f"guidance pairs x{world // 2} (eps all-gathered per step over NCCL)",
                   "timing": "CUDA-graph replay of the half forward, the pair's all-gather, the update"},
        "pair_latents_identical": bool(same.item() == 1.0),
        "clocks": clocks.summary(), "device_status": status,
    }
    print(json.dumps(line), flush=True)


def run_unet(args, torch, dev, dist, world, rank, local, barrier, max_over_ranks) -> None:
    import sdb
    import unet as U

    net = U.UNet(U.SD15, device=dev, seed=20261011)
    # This rank's images of the 8-image batch (one a rank past 8 GPUs).
    per = max(1, IMAGES // world)
    sampler = U.Sampler(net, 64, 64, steps=SAMPLER_STEPS, images=per)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    latent = torch.randn(per, 64, 64, 4, device=dev, generator=g)
    context = torch.randn(2 * per, 77, 768, device=dev, generator=g)
    sampler.x.copy_(latent * sampler.sigmas[0])
    sampler.context.copy_(context)
    sampler.set_step(0)
    n0 = sdb.launch_count()
    sampler.capture(warmup=max(3, args.warmup))
    launches_forward = sdb.launch_count() - n0
    # Per step on the device: the timestep, the captured forward, the guidance + Euler update (which
    # also writes the next step's model input).
    ts = torch.tensor([U.sigma_to_t(sg) for sg in sampler.sigmas[:-1]], device=dev, dtype=torch.float32)
    c_in = [1.0 / math.sqrt(sg * sg + 1.0) for sg in sampler.sigmas]

    def step(i: int) -> None:
        j = i % SAMPLER_STEPS
        sampler.t.copy_(ts[j:j + 1].expand(2 * per))
        eps = sampler.step_forward()
        sdb.euler_cfg_step(eps, sampler.x, sampler.x_in, sampler.cfg_scale, sampler.sigmas[j],
                           sampler.sigmas[j + 1], c_in[(j + 1) % SAMPLER_STEPS])

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    n0 = sdb.launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start.record()
        for i in range(args.steps):
            step(i)
        end.record()
        torch.cuda.synchronize()
    # Graph replays do not pass through the library's launch counter: the forward's launches times K,
    # plus the update kernel each step.
    launches = launches_forward // (max(3, args.warmup) + 1) * args.steps + (sdb.launch_count() - n0)
    barrier()
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)

    # The step's classes: the calls of one forward, each timed alone (graph replays).
    cap = torch.cuda.Stream(device=dev)
    cap.wait_stream(torch.cuda.current_stream())
    with OpClock(sdb, torch) as oc:
        with torch.cuda.stream(cap):
            net.forward(sampler.x_in, sampler.t, sampler.context)
    torch.cuda.synchronize()
    classes = oc.measure(cap)
    top_shapes = sorted(oc.shapes.items(), key=lambda kv: -kv[1][1])[:16]
    shapes = {k: {"ms": round(v[1], 4), "calls": v[2], "tflops": round(v[0] / (v[1] * 1e-3) / 1e12, 1)}
              for k, v in top_shapes}
    del oc

    # End to end through the public API: latent and context from pinned host memory, the sampler step,
    # the updated latent back to the host.
    h_lat = latent.cpu().pin_memory()
    h_ctx = context.cpu().pin_memory()
    h_out = torch.empty(per, 64, 64, 4).pin_memory()
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step(i: int) -> None:
        sampler.x.copy_(h_lat, non_blocking=True)
        sampler.context.copy_(h_ctx, non_blocking=True)
        step(i)
        h_out.copy_(sampler.x, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    e2e_step(0)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step(i)
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3 / e2e_steps)
    h2d = h_lat.numel() * 4 + h_ctx.numel() * 4
    d2h = h_out.numel() * 4
    # The VAE decode of this rank's latents, captured once and replayed.
    vae_ms, vae_flops = measure_vae(torch, dev, sampler.x, barrier, max_over_ranks)
    # The job's final latents to rank 0 (NCCL over NVLink): the gather benchmark config 4's image sharding
    # ends with, timed on the device as the max over ranks.
    gather = None
    if dist is not None and world > 1:
        lat_all = torch.empty(world * per, *sampler.x.shape[1:], device=dev) if rank == 0 else None
        for _ in range(2):
            dist.gather(sampler.x.contiguous(), [lat_all[i * per:(i + 1) * per] for i in range(world)]
                        if rank == 0 else None, dst=0)
        torch.cuda.synchronize()
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record()
        dist.gather(sampler.x.contiguous(), [lat_all[i * per:(i + 1) * per] for i in range(world)]
                    if rank == 0 else None, dst=0)
        g1.record()
        torch.cuda.synchronize()
        gather = {"ms": max_over_ranks(g0.elapsed_time(g1)), "bytes": world * sampler.x.numel() * 4,
                  "how": "torch.distributed.gather over NCCL of every rank's latents to rank 0"}
        del lat_all
    del sampler
    torch.cuda.empty_cache()
    # One image's latency: the same step on a CFG batch of 2 alone.
    ms1 = ms
    if per > 1:
        one = U.Sampler(net, 64, 64, steps=SAMPLER_STEPS, images=1)
        one.x.copy_(latent[:1] * one.sigmas[0])
        one.context.copy_(context[:2])
        one.set_step(0)
        one.capture(warmup=3)
        with torch.cuda.stream(torch.cuda.current_stream()):
            for _ in range(3):
                one.step_forward()
        barrier()
        torch.cuda.synchronize()
        s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s1.record()
        for i in range(10):
            one.t.copy_(ts[i:i + 1].expand(2))
            eps1 = one.step_forward()
            sdb.euler_cfg_step(eps1, one.x, one.x_in, one.cfg_scale, one.sigmas[i], one.sigmas[i + 1],
                               c_in[i + 1])
        e1.record()
        torch.cuda.synchronize()
        ms1 = max_over_ranks(s1.elapsed_time(e1) / 10)
        del one
        torch.cuda.empty_cache()
    sdxl = None if args.no_sdxl else measure_sdxl(torch, dev, barrier, max_over_ranks)
    status = sdb.device_status(clear=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    configs = hot_op_configs(torch, dev)
    peaks = measured_peaks()
    step_flops = net.flops(2 * per, 64, 64)
    dom = max((k for k in classes if CLASSES[k] == "tensor"), key=lambda k: classes[k]["ms"])
    d = classes[dom]
    achieved = d["work"] / (d["ms"] * 1e-3) / 1e12
    traffic = None
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.exists():
        # Captured on the UNet's launch of one image's guidance pair; DRAM bytes grow with the images a
        # launch processes (every launch streams its own activations), so scale by this GPU's images.
        traffic = json.loads(tfile.read_text()).get(dom)
        traffic = traffic * per if traffic is not None else None
    line = {
        "metric": UNET_METRIC, "value": world * per * 1e3 / ms, "unit": UNET_UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if world * per == IMAGES else "weak",
        "vs_baseline": None, "dtype": "f32" if not args.tune else f"f32 ({args.tune})", "data": "synthetic",
        "config": unet_config(world, args.tune),
        "unet_ms_per_step": ms,
        "unet_ms_per_step_one_image": ms1,
        "configs": configs,
        "latent_gather": gather,
        "vae_ms": vae_ms,
        "vae_tflops": vae_flops / (vae_ms * 1e-3) / 1e12,
        "imgs_per_s": world * per * 1e3 / (SAMPLER_STEPS * ms + vae_ms),
        "imgs_per_s_unet_only": world * per * 1e3 / ms / SAMPLER_STEPS,
        "sdxl": sdxl,
        "step_tflop": step_flops / 1e12,
        "step_frac_of_sustained_peak": step_flops / (ms * 1e-3) / 1e12 / peaks["bf16_tflops_sustained"],
        "roofline": {"kernel": f"{dom} (all calls of the class in one forward)", "bound": "tensor",
                     "achieved": achieved, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": achieved / peaks["bf16_tflops"], "peak_source": peaks["source"] + " (burst)",
                     "traffic": traffic, "work_per_launch": d["work"] / d["calls"],
                     "avg_launch_ms": d["ms"] / d["calls"]},
        "classes_ms": {k: round(v["ms"], 4) for k, v in sorted(classes.items(), key=lambda kv: -kv[1]["ms"])},
        "classes_tflops": {k: round(v["work"] / (v["ms"] * 1e-3) / 1e12, 1) for k, v in classes.items()
                           if CLASSES[k] == "tensor"},
        "top_shapes": shapes,
        "e2e": {"value": world * per * 1e3 / e2e_ms, "unit": UNET_UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "device_status": status,
    }
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_unet_step()
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        line["cpu_baseline"]["cpu"] = cb["cpu"]
        line["cpu_baseline"]["parts_s"] = cb["parts_s"]
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- ranks

def max_over_ranks(value: float, dist=None, device=None) -> float:
    """The largest of the ranks' values (the step time every rank reports): an all-reduce of one
    double, on `device` (the rank's GPU under NCCL, the CPU under gloo)."""
    if dist is None:
        return value
    import torch

    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- single operations for profiler captures

OPS = {
    # name: builder(torch, sdb, dev) -> callable running the operation once
    "conv3x3_320x64x64x2": lambda torch, sdb, dev: _op_conv(torch, sdb, dev, 320, 320, 64, 2),
    "conv3x3_1280x16x16x2": lambda torch, sdb, dev: _op_conv(torch, sdb, dev, 1280, 1280, 16, 2),
    "attention_4096x4096_d40_b1": lambda torch, sdb, dev: _op_attention(torch, sdb, dev, 4096, 4096, 40, 1),
    "attention_4096x77_d40_b2": lambda torch, sdb, dev: _op_attention(torch, sdb, dev, 4096, 77, 40, 2),
    "linear_8192x320x320": lambda torch, sdb, dev: _op_linear(torch, sdb, dev, 8192, 320, 320),
    "linear_8192x320x1280": lambda torch, sdb, dev: _op_linear(torch, sdb, dev, 8192, 320, 1280),
    "linear_2048x640x640": lambda torch, sdb, dev: _op_linear(torch, sdb, dev, 2048, 640, 640),
    "linear_65536x320x320": lambda torch, sdb, dev: _op_linear(torch, sdb, dev, 65536, 320, 320),
    "groupnorm_2x64x64x320": lambda torch, sdb, dev: _op_groupnorm(torch, sdb, dev, 2, 64, 320),
}


def _op_conv(torch, sdb, dev, ic, oc, hw, n):
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(n, hw, hw, ic, device=dev, generator=g)
    w = (torch.randn(oc, ic, 3, 3, device=dev, generator=g) / math.sqrt(9 * ic)).half()
    b = torch.randn(oc, device=dev, generator=g)
    y = torch.empty(n, hw, hw, oc, device=dev)
    return lambda: sdb.conv2d_nhwc(w, x, (1, 1), (1, 1), out=y, chain=sdb.Chain().add(b, [0, 0, 1, 0]))


def _op_attention(torch, sdb, dev, lq, lk, d, b):
    g = torch.Generator(device=dev).manual_seed(1)
    q = torch.randn(b, lq, 8 * d, device=dev, generator=g)
    k = torch.randn(b, lk, 8 * d, device=dev, generator=g)
    v = torch.randn(b, lk, 8 * d, device=dev, generator=g)
    o = torch.empty(b, lq, 8 * d, device=dev)
    return lambda: sdb.attention_heads(q, k, v, 8, 8, d ** -0.5, out=o)


def _op_linear(torch, sdb, dev, m, k, n):
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(m, k, device=dev, generator=g)
    w = (torch.randn(n, k, device=dev, generator=g) / math.sqrt(k)).half()
    b = torch.randn(n, device=dev, generator=g)
    y = torch.empty(m, n, device=dev)
    return lambda: sdb.mul_mat(w, x, y, chain=sdb.Chain().add(b))


def _op_groupnorm(torch, sdb, dev, n, hw, c):
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(n, hw, hw, c, device=dev, generator=g)
    gamma = torch.randn(c, device=dev, generator=g)
    beta = torch.randn(c, device=dev, generator=g)
    y = torch.empty_like(x)
    chain = sdb.Chain().mul(gamma, [0, 0, 1, 0]).add(beta, [0, 0, 1, 0]).silu()
    return lambda: sdb.group_norm_nhwc(x, 32, 1e-5, out=y, chain=chain)


def run_op(name: str, tune: str = "", reps: int = 3) -> None:
    """Runs one named operation `reps` times (for ncu captures of a single kernel on a small case)."""
    import torch
    import sdb

    dev = torch.device("cuda", 0)
    sdb.load()
    if tune:
        sdb.set_tuning(tune)
    fn = OPS[name](torch, sdb, dev)
    for _ in range(reps):
        fn()
    torch.cuda.synchronize()
    print(json.dumps({"op": name, "reps": reps, "device_status": sdb.device_status(clear=True)}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["unet", "hot_ops"], default="unet")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sdxl", action="store_true", help="skip the SDXL step (benchmark config 5) measured beside SD 1.5")
    ap.add_argument("--cfg-split", action="store_true",
                    help="split classifier-free guidance over GPU pairs (needs an even number of ranks)")
    ap.add_argument("--op", choices=sorted(OPS), help="run one operation three times (profiler captures) and exit")
    ap.add_argument("--tune", default="", help="sdb_set_tuning spec for the run, e.g. bits=8 (the quantized linear layers)")
    args = ap.parse_args()
    if args.op:
        run_op(args.op, args.tune)
        return
    if args.steps is None:
        args.steps = 100 if args.workload == "unet" else 1000
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

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    import sdb

    sdb.load()
    if args.tune:
        sdb.set_tuning(args.tune)

    def barrier():
        if dist is not None:
            dist.barrier()

    run = (run_cfg_split if args.cfg_split else run_unet) if args.workload == "unet" else run_hot_ops
    run(args, torch, dev, dist, world, rank, local, barrier, lambda v: max_over_ranks(v, dist, dev))


if __name__ == "__main__":
    main()
