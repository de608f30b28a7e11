"""Parity of the quantized linear layers (tuning bits = 2..8).

The cases are the reference's quantized ones (tests/ops_test.cc:857-905): the
linear layers of 256 rows and more, which are quantized, and of fewer, which
are not; the gated GELU; groups of 32, 128 and 256; weights of 7 bits and
inputs of 7.  Two bounds hold for each: the product is the reference's C++
form (quant.cc:113-166, restated in oracle/ref_forms.c) bit for bit -- the
integers are summed exactly and every FP32 operation of the fold is the
form's -- and its error against the exact product, relative to the
magnitudes, is within the reference's own bound for its quantized forms,
1e-2 with 8 bits of both operands, in proportion to 2/L + 1/W with fewer
(ops_test.cc:213-239).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
import ref_forms
from helpers import canary_like, cuda_tensor, host, rng

pytestmark = pytest.mark.gpu


def bound(bits: int = 8, input_bits: int = 8) -> float:
    levels, wmax = (1 << input_bits) - 1, (1 << (bits - 1)) - 1
    return 1e-2 * (2.0 / levels + 1.0 / wmax) / (2.0 / 255 + 1.0 / 127)


class tuned:
    """Tuning for the duration of a block, restored after."""

    def __init__(self, spec: str):
        self.spec = spec

    def __enter__(self):
        import sdb

        sdb.set_tuning(self.spec)

    def __exit__(self, *exc):
        import sdb

        sdb.set_tuning("bits=0,input_bits=8,group=64,weight_group=1,quantize=7")


def run_linear(cuda, k, n, m, batch, wtype, seed=None, bias=False):
    import sdb

    g = rng() if seed is None else rng(seed)
    w = oracle.uniform(g, (n, k), 0.25, wtype)
    x = oracle.uniform(g, (batch, m, k), 1.0)
    b = oracle.uniform(g, (n,), 1.0) if bias else None
    out = canary_like((batch, m, n), cuda)
    chain = sdb.Chain().add(cuda_tensor(b, cuda)) if bias else None
    sdb.mul_mat(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out, chain=chain)
    return w, x, b, host(out)


# (k, n, m, batch, weight dtype) -- ops_test.cc:859-867
QUANTIZED_CASES = [
    (320, 320, 512, 2, np.float16),
    (768, 1280, 300, 1, np.float16),
    (1280, 320, 256, 1, np.float16),
    (77, 100, 300, 1, np.float32),
    (300, 17, 131, 3, np.float16),
    (40, 2560, 296, 1, np.float32),
]


@pytest.mark.parametrize("k,n,m,batch,wtype", QUANTIZED_CASES)
def test_quantized_mul_mat_reference_cases(cuda, k, n, m, batch, wtype):
    with tuned("bits=8"):
        w, x, _, got = run_linear(cuda, k, n, m, batch, wtype)
    form = ref_forms.qmul_mat(w, x.reshape(-1, k)).reshape(batch, m, n)
    assert np.array_equal(got.view(np.uint32), form.view(np.uint32)), \
        f"{np.count_nonzero(got != form)} of {got.size} differ from the C++ form"
    exact, mag = oracle.mul_mat_exact(w, x)
    err = oracle.metric(got, exact, mag)
    assert err <= bound(), f"error {err:.3g}"


def test_fewer_rows_are_not_quantized(cuda):
    """154 rows (< 256): the product stays in single precision (mul_mat.cc:101-105)."""
    with tuned("bits=8"):
        w, x, _, got = run_linear(cuda, 768, 320, 77, 2, np.float16)
    exact, mag = oracle.mul_mat_exact(w, x)
    assert oracle.metric(got, exact, mag) <= oracle.K_B200


def test_quantized_bias_chain_and_residual(cuda):
    """The chain after the product, and a residual written in place (the product's sums start from it)."""
    import sdb

    g = rng(11)
    k, n, m = 640, 384, 300
    w = oracle.uniform(g, (n, k), 0.25, np.float16)
    x = oracle.uniform(g, (m, k), 1.0)
    b = oracle.uniform(g, (n,), 1.0)
    r = oracle.uniform(g, (m, n), 1.0)
    res = cuda_tensor(r, cuda)
    out = canary_like((m, n), cuda)
    with tuned("bits=8"):
        sdb.mul_mat(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out,
                    chain=sdb.Chain().add(cuda_tensor(b, cuda)).redirect(res, from_redirect=True))
    form = ref_forms.qmul_mat(w, x, y0=r) + b
    got = host(res)
    assert np.array_equal(got.view(np.uint32), form.astype(np.float32).view(np.uint32))
    exact, mag = oracle.mul_mat_exact(w, x)
    exact = exact + r + b
    mag = mag + np.abs(r) + np.abs(b)
    assert oracle.metric(got, exact, mag) <= bound()


@pytest.mark.parametrize("group", [32, 128, 256])
def test_quantized_groups(cuda, group):
    with tuned(f"bits=8,group={group}"):
        w, x, _, got = run_linear(cuda, 640, 384, 300, 1, np.float16, seed=group)
    form = ref_forms.qmul_mat(w, x.reshape(-1, 640), group=group).reshape(got.shape)
    assert np.array_equal(got.view(np.uint32), form.view(np.uint32))
    exact, mag = oracle.mul_mat_exact(w, x)
    assert oracle.metric(got, exact, mag) <= bound()


@pytest.mark.parametrize("bits,input_bits", [(7, 8), (8, 7)])
@pytest.mark.parametrize("k,n,wtype", [(640, 384, np.float16), (77, 100, np.float32)])
def test_quantized_narrow_integers(cuda, bits, input_bits, k, n, wtype):
    with tuned(f"bits={bits},input_bits={input_bits}"):
        w, x, _, got = run_linear(cuda, k, n, 300, 1, wtype, seed=bits * 10 + input_bits)
    form = ref_forms.qmul_mat(w, x.reshape(-1, k), levels=(1 << input_bits) - 1,
                              wmax=(1 << (bits - 1)) - 1).reshape(got.shape)
    assert np.array_equal(got.view(np.uint32), form.view(np.uint32))
    exact, mag = oracle.mul_mat_exact(w, x)
    assert oracle.metric(got, exact, mag) <= bound(bits, input_bits)


def test_quantized_row_scales(cuda):
    """weight_group=0: one scale for a whole row of k (benchmark config 5's weights)."""
    with tuned("bits=8,weight_group=0"):
        w, x, _, got = run_linear(cuda, 1280, 320, 300, 1, np.float16, seed=3)
    form = ref_forms.qmul_mat(w, x.reshape(-1, 1280), weight_groups=False).reshape(got.shape)
    assert np.array_equal(got.view(np.uint32), form.view(np.uint32))
    exact, mag = oracle.mul_mat_exact(w, x)
    assert oracle.metric(got, exact, mag) <= bound()


# (k, half, m, batch, tuning) -- ops_test.cc:871-884
GATED_CASES = [
    (320, 1280, 200, 2, "bits=8"),
    (96, 2000, 300, 1, "bits=8"),
    (256, 640, 300, 1, "bits=8,group=128"),
    (256, 640, 300, 1, "bits=8,group=32"),
    (256, 640, 300, 1, "bits=7"),
]


@pytest.mark.parametrize("k,half,m,batch,spec", GATED_CASES)
def test_quantized_gated(cuda, k, half, m, batch, spec):
    import sdb

    g = rng()
    w = oracle.uniform(g, (2 * half, k), 0.25, np.float16)
    x = oracle.uniform(g, (batch, m, k), 1.0)
    b = oracle.uniform(g, (2 * half,), 1.0)
    out = canary_like((batch, m, half), cuda)
    with tuned(spec):
        opts = dict(kv.split("=") for kv in spec.split(","))
        bits = int(opts.get("bits", 8))
        group = int(opts.get("group", 64))
        sdb.mul_mat_gated(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out, chain=sdb.Chain().add(cuda_tensor(b, cuda)))
    got = host(out)
    # The product is the C++ form's; the GELU after it is the FP32 one of the single-precision path.
    y = ref_forms.qmul_mat(w, x.reshape(-1, k), group=group, wmax=(1 << (bits - 1)) - 1) + b
    want = (y[:, :half] * oracle.gelu(y[:, half:])).reshape(got.shape)
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=2e-6 * np.abs(want).max())
    exact, mag = oracle.gated_exact(w, x, b)
    assert oracle.metric(got, exact, mag) <= bound(bits)


def test_quantized_gated_half_not_a_panel(cuda):
    """Quantized, a half of no multiple of 16 is not fused (mul_mat.cc:1130-1133): the caller splits it."""
    import sdb
    import torch

    w = torch.zeros(200, 40, dtype=torch.float16, device=cuda)
    x = torch.zeros(300, 40, device=cuda)
    out = torch.zeros(300, 100, device=cuda)
    with tuned("bits=8"):
        assert not sdb.mul_mat_gated_supported(w, x, out)
    assert sdb.mul_mat_gated_supported(w, x, out)


def test_quantized_weights_kept_per_variant(cuda):
    """The store keeps one quantized form per variant (group, bits, weight_group) and the FP16 panels apart."""
    import sdb

    g = rng(5)
    w = cuda_tensor(oracle.uniform(g, (256, 320), 0.25, np.float16), cuda)
    x = cuda_tensor(oracle.uniform(g, (300, 320), 1.0), cuda)
    sdb.forget(w)
    e0, _ = sdb.store_stats()
    outs = []
    for spec in ("bits=8", "bits=8,group=32", "bits=8", "bits=0"):
        with tuned(spec):
            outs.append(host(sdb.mul_mat(w, x)))
    e1, _ = sdb.store_stats()
    assert e1 - e0 == 3
    assert np.array_equal(outs[0], outs[2])
    assert not np.array_equal(outs[0], outs[1])
