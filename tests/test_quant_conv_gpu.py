"""Parity of the quantized convolutions (tuning bits = 2..8, quantize's convolution bit).

The reference computes a quantized convolution in one of two forms, by its own
rule (winograd.cc:2107-2123): Winograd's F(2x2, 3x3) with the xi products in
integers for 3x3 kernels at stride 1 of at least winograd_positions outputs an
image or at most winograd_small_tiles tiles in all; every other convolution
directly, the columns of each output position quantized in groups of
K = (ic, ky, kx) (conv2d.cc:338-470).  The cases are the reference's quantized
conv list (ops_test.cc:841-853), which takes both, its narrower integers
(ops_test.cc:896-903), and the chains and layouts this build adds.

Two bounds hold for each, as for the quantized linear layers: the result is the
reference's C++ form bit for bit (oracle/ref_forms.py qconv2d, qwinograd2: the
transforms in the reference's order of FP32 operations, the integer sums exact,
the fold's FP32 arithmetic the form's), and its error against the exact
convolution, relative to the magnitudes, is within the reference's bound for
quantized forms (ops_test.cc:213-239).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import ref_forms
from helpers import canary_like, cuda_tensor, host, rng
from test_quant_gpu import bound, tuned

pytestmark = pytest.mark.gpu

# (w, h, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1, n, weight dtype): ops_test.cc:843-852.
CASES = [
    (64, 64, 64, 48, 3, 3, 1, 1, 1, 1, 1, 1, 2, np.float16),
    (16, 16, 96, 64, 3, 3, 1, 1, 1, 1, 1, 1, 2, np.float16),
    (8, 8, 96, 64, 3, 3, 1, 1, 1, 1, 1, 1, 2, np.float16),
    (32, 32, 64, 40, 1, 1, 1, 1, 0, 0, 1, 1, 2, np.float16),
    (33, 33, 24, 30, 3, 3, 2, 2, 1, 1, 1, 1, 1, np.float16),
    (17, 13, 5, 7, 3, 3, 1, 1, 1, 1, 1, 1, 3, np.float32),
    (65, 33, 24, 20, 3, 3, 1, 1, 1, 1, 1, 1, 2, np.float16),
    (64, 20, 13, 11, 3, 3, 1, 1, 0, 0, 1, 1, 1, np.float16),
    (96, 16, 32, 17, 3, 3, 1, 1, 1, 1, 1, 1, 1, np.float32),
]


def ids(c):
    return "x".join(map(str, c[:4])) + f"_k{c[4]}s{c[6]}p{c[8]}{c[9]}_n{c[12]}_{np.dtype(c[13]).name}"


def winograd_taken(case, positions=1024, small_tiles=256) -> bool:
    """The reference's choice of form for a quantized convolution (winograd.cc:2107-2123, 194-196)."""
    wd, h, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1, n, _ = case
    if (kw, kh, s0, s1, d0, d1) != (3, 3, 1, 1, 1, 1) or not (0 <= p0 <= 2 and 0 <= p1 <= 2):
        return False
    ow, oh = wd + 2 * p0 - 2, h + 2 * p1 - 2
    return ow * oh >= positions or n * ((ow + 1) // 2) * ((oh + 1) // 2) <= small_tiles


def form(case, w, x, group=64, levels=255, wmax=127, weight_groups=True, span=None):
    wd, h, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1, n, _ = case
    if winograd_taken(case):
        return ref_forms.qwinograd2(w, x, (p0, p1), group, levels, wmax, weight_groups, span)
    return ref_forms.qconv2d(w, x, (s0, s1), (p0, p1), (d0, d1), group, levels, wmax, weight_groups)


def run(cuda, case, seed=None, chain=None, out=None):
    import sdb

    wd, h, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1, n, wtype = case
    g = rng() if seed is None else rng(seed)
    w = oracle.uniform(g, (oc, ic, kh, kw), 0.25, wtype)
    x = oracle.uniform(g, (n, ic, h, wd), 1.0)
    oh = (h + 2 * p1 - d1 * (kh - 1) - 1) // s1 + 1
    ow = (wd + 2 * p0 - d0 * (kw - 1) - 1) // s0 + 1
    out = canary_like((n, oc, oh, ow), cuda) if out is None else out
    sdb.conv2d(cuda_tensor(w, cuda), cuda_tensor(x, cuda), (s0, s1), (p0, p1), (d0, d1), out=out, chain=chain)
    return w, x, host(out)


def check(got, want, w, x, case, bits=8, input_bits=8):
    wd, h, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1, n, _ = case
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{np.count_nonzero(got != want)} of {got.size} differ from the C++ form"
    exact, mag = oracle.conv2d_exact(w, x, (s0, s1), (p0, p1), (d0, d1))
    err = oracle.metric(got, exact, mag)
    assert err <= bound(bits, input_bits), f"error {err:.3g}"


@pytest.mark.parametrize("case", CASES, ids=ids)
def test_quantized_conv_reference_cases(cuda, case):
    with tuned("bits=8"):
        w, x, got = run(cuda, case)
    check(got, form(case, w, x), w, x, case)


NARROW = [CASES[0], CASES[4], CASES[5]]  # ops_test.cc:900-902


@pytest.mark.parametrize("bits,input_bits", [(7, 8), (8, 7)])
@pytest.mark.parametrize("case", NARROW, ids=ids)
def test_quantized_conv_narrow_integers(cuda, case, bits, input_bits):
    with tuned(f"bits={bits},input_bits={input_bits}"):
        w, x, got = run(cuda, case)
    want = form(case, w, x, levels=(1 << input_bits) - 1, wmax=(1 << (bits - 1)) - 1)
    check(got, want, w, x, case, bits, input_bits)


@pytest.mark.parametrize("group", [32, 128, 256])
@pytest.mark.parametrize("case", [CASES[0], CASES[3]], ids=ids)
def test_quantized_conv_groups(cuda, case, group):
    with tuned(f"bits=8,group={group}"):
        w, x, got = run(cuda, case)
    check(got, form(case, w, x, group=group), w, x, case)


# Per-row weight scales: over the whole of K directly; over the reference's stretch of input channels
# for Winograd -- 256 of the 320 for many tiles, 128 for few (winograd.cc:238-268).
ROW_SCALE_CASES = [
    ((40, 40, 320, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1, np.float16), 256),
    ((12, 12, 320, 72, 3, 3, 1, 1, 1, 1, 1, 1, 2, np.float16), 128),
    ((20, 20, 320, 48, 3, 3, 2, 2, 1, 1, 1, 1, 1, np.float16), None),
]


@pytest.mark.parametrize("case,span", ROW_SCALE_CASES, ids=lambda v: ids(v) if isinstance(v, tuple) else str(v))
def test_quantized_conv_row_scales(cuda, case, span):
    with tuned("bits=8,weight_group=0"):
        w, x, got = run(cuda, case)
    check(got, form(case, w, x, weight_groups=False, span=span), w, x, case)


@pytest.mark.parametrize("case", [CASES[0], CASES[1], CASES[4]], ids=ids)
def test_quantized_conv_bias_residual(cuda, case):
    """conv + bias + residual, the sum begun from the residual in its own memory (redirect): Winograd
    adds it to each output of A^T M A (winograd.cc:543-575), the direct form begins its fold from it;
    then the bias."""
    import sdb

    wd, h, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1, n, wtype = case
    oh = (h + 2 * p1 - d1 * (kh - 1) - 1) // s1 + 1
    ow = (wd + 2 * p0 - d0 * (kw - 1) - 1) // s0 + 1
    g = rng(41)
    b = oracle.uniform(g, (1, oc, 1, 1), 1.0)
    r = oracle.uniform(g, (n, oc, oh, ow), 1.0)
    out = cuda_tensor(r, cuda).clone()
    scratch = canary_like((n, oc, oh, ow), cuda)
    with tuned("bits=8"):
        w, x, _ = run(cuda, case, chain=sdb.Chain().add(cuda_tensor(b, cuda)).redirect(out, from_redirect=True),
                      out=scratch)
        got = host(out)
    if winograd_taken(case):
        want = (r + form(case, w, x)) + b
    else:
        # The direct form's fold starts from the residual itself (quant.cc:113-166, accumulate).
        cols, _ = ref_forms.im2col(x, kh, kw, (s0, s1), (p0, p1), (d0, d1))
        y0 = r.transpose(0, 2, 3, 1).reshape(-1, oc)
        want = ref_forms.qmul_mat(w.astype(np.float32).reshape(oc, -1), cols, y0=y0)
        want = want.reshape(n, oh, ow, oc).transpose(0, 3, 1, 2) + b
    assert np.array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32)), \
        f"{np.count_nonzero(got != want)} of {got.size} differ from the C++ form"


@pytest.mark.parametrize("case", [CASES[0], CASES[3], CASES[4]], ids=ids)
def test_quantized_conv_channels_last(cuda, case):
    """Channels-last image in and out (the UNet runner's layout) with a bias: the same bits."""
    import sdb
    import torch

    wd, h, ic, oc, kw, kh, s0, s1, p0, p1, d0, d1, n, wtype = case
    oh = (h + 2 * p1 - d1 * (kh - 1) - 1) // s1 + 1
    ow = (wd + 2 * p0 - d0 * (kw - 1) - 1) // s0 + 1
    g = rng(42)
    w = oracle.uniform(g, (oc, ic, kh, kw), 0.25, wtype)
    x = oracle.uniform(g, (n, ic, h, wd), 1.0)
    b = oracle.uniform(g, (oc,), 1.0)
    xt = cuda_tensor(x, cuda).permute(0, 2, 3, 1).contiguous()
    out = torch.full((n, oh, ow, oc), float("nan"), device=cuda)
    with tuned("bits=8"):
        sdb.conv2d_nhwc(cuda_tensor(w, cuda), xt, (s0, s1), (p0, p1), (d0, d1), out=out,
                        chain=sdb.Chain().add(cuda_tensor(b, cuda), sdb.channel_operand(None)))
    got = np.ascontiguousarray(host(out).transpose(0, 3, 1, 2))
    want = form(case, w, x) + b.reshape(1, oc, 1, 1)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"{np.count_nonzero(got != want)} of {got.size} differ from the C++ form"


def test_quantized_conv_weights_kept_per_variant(cuda):
    """The store keeps one quantized packing per variant (group, bits, scale span) and reuses it."""
    import sdb

    case = CASES[0]
    g = rng(43)
    wd, h, ic, oc = case[:4]
    w = cuda_tensor(oracle.uniform(g, (oc, ic, 3, 3), 0.25, np.float16), cuda)
    x = cuda_tensor(oracle.uniform(g, (2, ic, h, wd), 1.0), cuda)
    sdb.forget(w)
    e0, _ = sdb.store_stats()
    with tuned("bits=8"):
        y1 = sdb.conv2d(w, x, (1, 1), (1, 1), (1, 1))
        y2 = sdb.conv2d(w, x, (1, 1), (1, 1), (1, 1))
        assert sdb.store_stats()[0] == e0 + 1
    with tuned("bits=8,group=128"):
        sdb.conv2d(w, x, (1, 1), (1, 1), (1, 1))
        assert sdb.store_stats()[0] == e0 + 2
    assert bool((y1 == y2).all())
    sdb.forget(w)
    assert sdb.store_stats()[0] == e0
