"""Parity of Winograd's F(2x2, 3x3) and F(4x4, 3x3) convolutions against the exact oracle.

Cases: every 3x3, stride-1 case of the reference's conv list (ops_test.cc:801-819)
in both forms, with the position thresholds lowered so each takes Winograd; the
chains the reference's fusion tests put after a Winograd convolution (bias and
residual, residual in its own memory: ops_test.cc:976-1066); channels-last images;
benchmark config 2's shapes under the default tuning.

Bounds (ops_test metric, error over the summed product magnitudes):
  F(2x2): <= 1e-6;
  F(4x4): <= max(1e-6, 1.5 x the error of the reference's single-precision F(4x4)
          form on the same inputs, oracle.winograd_f32) -- F(4x4)'s transforms
          round about seven times as much as F(2x2)'s (winograd.cc:1165-1168),
          and that, not the product split, sets its error.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from helpers import canary_like, cuda_tensor, host, rng

pytestmark = pytest.mark.gpu

# (w, h, ic, oc, p0, p1, n, weight dtype): the 3x3 stride-1 cases of ops_test.cc:801-819.
CASES = [
    (64, 64, 64, 48, 1, 1, 2, np.float16),
    (16, 16, 96, 64, 1, 1, 2, np.float16),
    (8, 8, 96, 64, 1, 1, 2, np.float16),
    (17, 13, 5, 7, 1, 1, 3, np.float32),
    (100, 3, 20, 25, 0, 1, 1, np.float16),
    (512, 4, 16, 3, 1, 1, 1, np.float16),
    (65, 33, 24, 20, 1, 1, 2, np.float16),
    (64, 20, 13, 11, 0, 0, 1, np.float16),
    (96, 16, 32, 17, 1, 1, 1, np.float32),
    (128, 128, 8, 8, 1, 1, 1, np.float16),
    # padding 2 (the reference takes 0..2)
    (20, 18, 24, 40, 2, 2, 1, np.float16),
]

FORCE = "winograd_positions=0,winograd4_positions=0,winograd_channels=0"
DEFAULT = "winograd=2,winograd_positions=1024,winograd4_positions=256,winograd_channels=16"


def ids(c):
    return "x".join(map(str, c[:4])) + f"_p{c[4]}{c[5]}_n{c[6]}_{np.dtype(c[7]).name}"


def bound(f: int, w, x, pad, exact, mag) -> float:
    if f != 4:
        return oracle.K_B200
    ref = oracle.metric(oracle.winograd_f32(w, x, pad, 4), exact, mag)
    return max(oracle.K_B200, 1.5 * ref)


@pytest.mark.parametrize("form", [1, 2], ids=["F2", "F4"])
@pytest.mark.parametrize("case", CASES, ids=ids)
def test_winograd_cases(cuda, case, form):
    import sdb

    wd, h, ic, oc, p0, p1, n, wtype = case
    g = rng()
    w = oracle.uniform(g, (oc, ic, 3, 3), 0.25, wtype)
    x = oracle.uniform(g, (n, ic, h, wd), 1.0)
    out = canary_like((n, oc, h + 2 * p1 - 2, wd + 2 * p0 - 2), cuda)
    sdb.set_tuning(f"winograd={form},{FORCE}")
    try:
        sdb.conv2d(cuda_tensor(w, cuda), cuda_tensor(x, cuda), (1, 1), (p0, p1), (1, 1), out=out)
    finally:
        sdb.set_tuning(DEFAULT)
    exact, mag = oracle.conv2d_exact(w, x, (1, 1), (p0, p1), (1, 1))
    # F(4x4) takes FP16 kernels of 16 input channels and more; the rest F(2x2).
    f = 4 if form == 2 and wtype == np.float16 and ic >= 16 else 2
    err = oracle.metric(host(out), exact, mag)
    assert err <= bound(f, w, x, (p0, p1), exact, mag), f"F({f}x{f}) error {err:.3g}"


@pytest.mark.parametrize("form", [1, 2], ids=["F2", "F4"])
@pytest.mark.parametrize("residual", ["in_place", "own_memory"])
def test_winograd_bias_residual(cuda, form, residual):
    """conv + bias + residual (ops_test.cc:976-1066): the residual added in place after
    the bias, or the sum begun from the residual in its own memory (redirect)."""
    import sdb

    g = rng(7)
    n, ic, oc, h, wd = 2, 40, 24, 24, 20
    w = oracle.uniform(g, (oc, ic, 3, 3), 0.25, np.float16)
    x = oracle.uniform(g, (n, ic, h, wd), 1.0)
    b = oracle.uniform(g, (1, oc, 1, 1), 1.0)
    r = oracle.uniform(g, (n, oc, h, wd), 1.0)
    bt, rt = cuda_tensor(b, cuda), cuda_tensor(r, cuda)
    sdb.set_tuning(f"winograd={form},{FORCE}")
    try:
        if residual == "in_place":
            out = canary_like((n, oc, h, wd), cuda)
            sdb.conv2d(cuda_tensor(w, cuda), cuda_tensor(x, cuda), (1, 1), (1, 1), (1, 1), out=out,
                       chain=sdb.Chain().add(bt).add(rt))
        else:
            scratch = canary_like((n, oc, h, wd), cuda)
            out = rt.clone()
            sdb.conv2d(cuda_tensor(w, cuda), cuda_tensor(x, cuda), (1, 1), (1, 1), (1, 1), out=scratch,
                       chain=sdb.Chain().add(bt).redirect(out, from_redirect=True))
    finally:
        sdb.set_tuning(DEFAULT)
    exact, mag = oracle.conv2d_exact(w, x, (1, 1), (1, 1), (1, 1))
    exact = exact + b + r
    mag = mag + np.abs(b) + np.abs(r)
    f = 4 if form == 2 else 2
    err = oracle.metric(host(out), exact, mag)
    assert err <= bound(f, w, x, (1, 1), exact, mag), f"error {err:.3g}"


@pytest.mark.parametrize("form", [1, 2], ids=["F2", "F4"])
def test_winograd_channels_last_silu(cuda, form):
    """A channels-last image in and out (the UNet runner's layout), with bias then SiLU."""
    import sdb
    import torch

    g = rng(8)
    n, ic, oc, h, wd = 2, 64, 72, 32, 36
    w = oracle.uniform(g, (oc, ic, 3, 3), 0.25, np.float16)
    x = oracle.uniform(g, (n, ic, h, wd), 1.0)
    b = oracle.uniform(g, (oc,), 1.0)
    xt = cuda_tensor(x, cuda).permute(0, 2, 3, 1).contiguous()
    out = torch.full((n, h, wd, oc), float("nan"), device=cuda)
    sdb.set_tuning(f"winograd={form},{FORCE}")
    try:
        sdb.conv2d_nhwc(cuda_tensor(w, cuda), xt, (1, 1), (1, 1), (1, 1), out=out,
                        chain=sdb.Chain().add(cuda_tensor(b, cuda), sdb.channel_operand(None)).silu())
    finally:
        sdb.set_tuning(DEFAULT)
    got = host(out).transpose(0, 3, 1, 2)
    exact, mag = oracle.conv2d_exact(w, x, (1, 1), (1, 1), (1, 1))
    pre = exact + b.reshape(1, oc, 1, 1)
    want = pre / (1 + np.exp(-pre))
    # SiLU's slope is at most 1.1: the pre-activation bound carries over.
    f = 4 if form == 2 else 2
    err = oracle.metric(got, want, mag + np.abs(b.reshape(1, oc, 1, 1)))
    assert err <= 1.1 * bound(f, w, x, (1, 1), exact, mag) + 2e-7, f"error {err:.3g}"


CONFIG2 = [(320, 64), (640, 32), (1280, 8)]


@pytest.mark.parametrize("c,hw", CONFIG2, ids=lambda v: str(v))
def test_winograd_config2_default(cuda, c, hw):
    """benchmark config 2 under the default tuning (Winograd where it is taken) with its bias."""
    import sdb

    g = rng(20)
    x = g.standard_normal((1, c, hw, hw)).astype(np.float32)
    w = (g.standard_normal((c, c, 3, 3)) / np.sqrt(9 * c)).astype(np.float32).astype(np.float16)
    b = (g.standard_normal(c) * 0.02).astype(np.float32)
    out = canary_like((1, c, hw, hw), cuda)
    bt = cuda_tensor(b.reshape(1, c, 1, 1), cuda)
    sdb.set_tuning(DEFAULT)
    sdb.conv2d(cuda_tensor(w, cuda), cuda_tensor(x, cuda), (1, 1), (1, 1), (1, 1), out=out, chain=sdb.Chain().add(bt))
    exact0, mag0 = oracle.conv2d_exact(w, x, (1, 1), (1, 1), (1, 1))
    exact = exact0 + b.reshape(1, c, 1, 1).astype(np.float64)
    mag = mag0 + np.abs(b.reshape(1, c, 1, 1).astype(np.float64))
    err = oracle.metric(host(out), exact, mag)
    f = 4 if hw * hw >= 1024 else 0
    assert err <= bound(f, w, x, (1, 1), exact0, mag0), f"error {err:.3g}"


def test_winograd_weights_kept_and_forgotten(cuda):
    """The transformed kernels are kept by the store (one entry per form) and dropped by forget."""
    import sdb

    g = rng(9)
    w = cuda_tensor(oracle.uniform(g, (32, 16, 3, 3), 0.25, np.float16), cuda)
    x = cuda_tensor(oracle.uniform(g, (1, 16, 40, 40), 1.0), cuda)
    sdb.forget(w)
    e0, _ = sdb.store_stats()
    sdb.set_tuning(f"winograd=2,{FORCE}")
    try:
        y1 = sdb.conv2d(w, x, (1, 1), (1, 1), (1, 1))
        y2 = sdb.conv2d(w, x, (1, 1), (1, 1), (1, 1))
        e1, _ = sdb.store_stats()
        assert e1 == e0 + 1
        assert bool((y1 == y2).all())
        # A changed weight, forgotten, is transformed anew.
        w.mul_(-1.0)
        sdb.forget(w)
        y3 = sdb.conv2d(w, x, (1, 1), (1, 1), (1, 1))
    finally:
        sdb.set_tuning(DEFAULT)
    assert bool((y3 == -y1).all())
