"""Parity of the direct and Winograd convolutions against the exact oracle.

Cases: the reference's 13 (tests/ops_test.cc:801-819) -- the UNet's 3x3
convolutions made smaller, 1x1, stride 2, odd edges, FP32 weights, a 5x3
kernel with dilation -- each in every form the tuning offers (direct,
F(2x2), F(4x4)), and the three benchmark config 2 shapes.  Bound: the ops_test
metric <= 1e-6.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from helpers import canary_like, cuda_tensor, host, rng

pytestmark = pytest.mark.gpu

# (w, h, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1, n, weight dtype) -- ops_test.cc:801-819
CONV_CASES = [
    (64, 64, 64, 48, 3, 3, 1, 1, 1, 1, 1, 1, 2, np.float16),
    (16, 16, 96, 64, 3, 3, 1, 1, 1, 1, 1, 1, 2, np.float16),
    (8, 8, 96, 64, 3, 3, 1, 1, 1, 1, 1, 1, 2, np.float16),
    (32, 32, 64, 40, 1, 1, 1, 1, 0, 0, 1, 1, 2, np.float16),
    (33, 33, 24, 30, 3, 3, 2, 2, 1, 1, 1, 1, 1, np.float16),
    (17, 13, 5, 7, 3, 3, 1, 1, 1, 1, 1, 1, 3, np.float32),
    (40, 9, 7, 13, 5, 3, 1, 2, 2, 0, 2, 1, 1, np.float32),
    (100, 3, 20, 25, 3, 3, 1, 1, 0, 1, 1, 1, 1, np.float16),
    (512, 4, 16, 3, 3, 3, 1, 1, 1, 1, 1, 1, 1, np.float16),
    (65, 33, 24, 20, 3, 3, 1, 1, 1, 1, 1, 1, 2, np.float16),
    (64, 20, 13, 11, 3, 3, 1, 1, 0, 0, 1, 1, 1, np.float16),
    (96, 16, 32, 17, 3, 3, 1, 1, 1, 1, 1, 1, 1, np.float32),
    (128, 128, 8, 8, 3, 3, 1, 1, 1, 1, 1, 1, 1, np.float16),
]


def run_case(cuda, case, winograd: int):
    import sdb

    wd, h, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1, n, wtype = case
    g = rng()
    w = oracle.uniform(g, (oc, ic, kh, kw), 0.25, wtype)
    x = oracle.uniform(g, (n, ic, h, wd), 1.0)
    oh = oracle.conv_out(h, kh, s1, p1, d1)
    ow = oracle.conv_out(wd, kw, s0, p0, d0)
    out = canary_like((n, oc, oh, ow), cuda)
    sdb.set_tuning(f"winograd={winograd}")
    try:
        sdb.conv2d(cuda_tensor(w, cuda), cuda_tensor(x, cuda), (s0, s1), (p0, p1), (d0, d1), out=out)
    finally:
        sdb.set_tuning("winograd=2")
    exact, mag = oracle.conv2d_exact(w, x, (s0, s1), (p0, p1), (d0, d1))
    return oracle.metric(host(out), exact, mag)


@pytest.mark.parametrize("case", CONV_CASES, ids=lambda c: "x".join(map(str, c[:4])) + f"_k{c[5]}{c[4]}_s{c[6]}")
def test_conv2d_direct(cuda, case):
    err = run_case(cuda, case, 0)
    assert err <= oracle.K_B200, f"error {err:.3g}"


# benchmark config 2: 3x3, stride 1, pad 1, FP16 weights N(0, 1/sqrt(9 Cin)),
# FP32 input N(0, 1), bias, then GroupNorm(32, eps 1e-5, gamma ~ N(1, 0.1),
# beta ~ N(0, 0.1)), then SiLU.
CONFIG2 = [(320, 64), (640, 32), (1280, 8)]


@pytest.mark.parametrize("c,hw", CONFIG2, ids=lambda v: str(v))
def test_conv2d_config2(cuda, c, hw):
    """The convolution with its bias, against the exact oracle (ops_test metric <= 1e-6)."""
    import sdb

    g = rng(20)
    x = g.standard_normal((1, c, hw, hw)).astype(np.float32)
    w = (g.standard_normal((c, c, 3, 3)) / np.sqrt(9 * c)).astype(np.float32).astype(np.float16)
    b = (g.standard_normal(c) * 0.02).astype(np.float32)
    out = canary_like((1, c, hw, hw), cuda)
    bt = cuda_tensor(b.reshape(1, c, 1, 1), cuda)
    sdb.conv2d(cuda_tensor(w, cuda), cuda_tensor(x, cuda), (1, 1), (1, 1), (1, 1), out=out, chain=sdb.Chain().add(bt))
    exact, mag = oracle.conv2d_exact(w, x, (1, 1), (1, 1), (1, 1))
    exact = exact + b.reshape(1, c, 1, 1).astype(np.float64)
    mag = mag + np.abs(b.reshape(1, c, 1, 1).astype(np.float64))
    err = oracle.metric(host(out), exact, mag)
    assert err <= oracle.K_B200, f"error {err:.3g}"


@pytest.mark.parametrize("form", ["direct", "default"])
@pytest.mark.parametrize("c,hw", CONFIG2, ids=lambda v: str(v))
def test_conv_bias_groupnorm_silu_config2(cuda, c, hw, form):
    """The whole config-2 sequence (conv + bias, GroupNorm + gamma + beta + SiLU) against
    the same sequence in double precision.  Direct convolution: within 1e-6 of the
    largest output.  Default tuning (F(4x4) at 64x64 and 32x32, as the reference):
    within 1e-6 of the largest output or 1.5x the error of the reference's own
    single-precision F(4x4) form (oracle.winograd_f32) carried through the same
    GroupNorm and SiLU, whichever is larger -- GroupNorm divides by the group's
    deviation, which F(4x4)'s transform rounding does not shrink."""
    import sdb

    sdb.set_tuning("winograd=0" if form == "direct" else "winograd=2")
    try:
        _config2_sequence(cuda, c, hw, form)
    finally:
        sdb.set_tuning("winograd=2")


def _config2_sequence(cuda, c, hw, form):
    import sdb

    g = rng(21)
    x = g.standard_normal((1, c, hw, hw)).astype(np.float32)
    w = (g.standard_normal((c, c, 3, 3)) / np.sqrt(9 * c)).astype(np.float32).astype(np.float16)
    b = (g.standard_normal(c) * 0.02).astype(np.float32)
    gamma = (1 + 0.1 * g.standard_normal(c)).astype(np.float32)
    beta = (0.1 * g.standard_normal(c)).astype(np.float32)
    bt = cuda_tensor(b.reshape(1, c, 1, 1), cuda)
    y = sdb.conv2d(cuda_tensor(w, cuda), cuda_tensor(x, cuda), (1, 1), (1, 1), (1, 1), chain=sdb.Chain().add(bt))
    chain = sdb.Chain().mul(cuda_tensor(gamma.reshape(1, c, 1, 1), cuda)).add(
        cuda_tensor(beta.reshape(1, c, 1, 1), cuda)).silu()
    out = sdb.group_norm(y, 32, 1e-5, chain=chain)
    exact, _ = oracle.conv2d_exact(w, x, (1, 1), (1, 1), (1, 1))
    exact = exact + b.reshape(1, c, 1, 1)
    z = oracle.group_norm_exact(exact, 32, 1e-5) * gamma.reshape(1, c, 1, 1) + beta.reshape(1, c, 1, 1)
    z = z / (1 + np.exp(-z))
    got = host(out).astype(np.float64)
    limit = 1e-6 * np.abs(z).max()
    if form == "default" and hw * hw >= 1024:
        ref = oracle.winograd_f32(w, x, (1, 1), 4).astype(np.float64) + b.reshape(1, c, 1, 1)
        zr = oracle.group_norm_exact(ref, 32, 1e-5) * gamma.reshape(1, c, 1, 1) + beta.reshape(1, c, 1, 1)
        zr = zr / (1 + np.exp(-zr))
        limit = max(limit, 1.5 * np.abs(zr - z).max())
    assert np.abs(got - z).max() <= limit


@pytest.mark.parametrize("n,h,wd,ic,oc", [(2, 16, 16, 320, 640), (1, 9, 7, 36, 20), (3, 8, 8, 64, 30)])
def test_conv1x1_channels_last_as_linear(cuda, n, h, wd, ic, oc):
    """A 1x1 convolution over channels-last images (the UNet's skip and projection convolutions):
    taken as a linear layer over the positions, with a per-channel bias, a residual in its own
    channels-last memory and SiLU, against float64."""
    import sdb
    import torch

    g = rng(ic + oc)
    w = oracle.uniform(g, (oc, ic, 1, 1), 0.25, np.float16)
    x = oracle.uniform(g, (n, ic, h, wd), 1.0)
    b = oracle.uniform(g, (oc,), 1.0)
    res = oracle.uniform(g, (n, oc, h, wd), 1.0)
    xt = cuda_tensor(x, cuda).permute(0, 2, 3, 1).contiguous()
    rt = cuda_tensor(res, cuda).permute(0, 2, 3, 1).contiguous()
    out = torch.full((n, h, wd, oc), float("nan"), device=cuda)
    chain = (sdb.Chain().add(cuda_tensor(b, cuda), sdb.channel_operand(None))
             .add(rt, [oc, wd * oc, 1, h * wd * oc]).silu())
    sdb.conv2d_nhwc(cuda_tensor(w, cuda), xt, (1, 1), (0, 0), (1, 1), out=out, chain=chain)
    assert sdb.device_status(clear=True) == 0
    got = host(out).transpose(0, 3, 1, 2)
    exact, mag = oracle.conv2d_exact(w, x, (1, 1), (0, 0), (1, 1))
    pre = exact + b.reshape(1, oc, 1, 1).astype(np.float64) + res.astype(np.float64)
    want = pre / (1 + np.exp(-pre))
    # SiLU's slope is at most 1.1: the pre-activation bound carries over.
    err = oracle.metric(got, want, mag + np.abs(b.reshape(1, oc, 1, 1)) + np.abs(res))
    assert err <= 1.1 * oracle.K_B200, f"error {err:.3g}"
