"""Parity of the linear layers (MUL_MAT, GEGLU) against the exact oracle.

The cases are the reference's (tests/ops_test.cc:825-832 for mul_mat,
:946-949 for the gated GELU) plus benchmark config 1 (4096 x 320 -> 1280 with
its bias).  Weights U(-0.25, 0.25), inputs U(-1, 1) (ops_test.cc:441-444);
every output starts as the NaN canary.  The bound is the north star's: the
ops_test metric (error / sum of |products|, against float64) <= 1e-6.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from helpers import canary_like, cuda_tensor, host, rng

pytestmark = pytest.mark.gpu

# (k, n, m, batch, weight dtype) -- ops_test.cc:825-832
MUL_MAT_CASES = [
    (320, 320, 512, 2, np.float16),
    (768, 1280, 77, 2, np.float16),
    (1280, 320, 64, 1, np.float16),
    (77, 100, 23, 1, np.float32),
    (300, 17, 31, 3, np.float16),
    (40, 2560, 96, 1, np.float32),
]


@pytest.mark.parametrize("k,n,m,batch,wtype", MUL_MAT_CASES)
def test_mul_mat_reference_cases(cuda, k, n, m, batch, wtype):
    import sdb

    g = rng()
    w = oracle.uniform(g, (n, k), 0.25, wtype)
    x = oracle.uniform(g, (batch, m, k), 1.0)
    out = canary_like((batch, m, n), cuda)
    sdb.mul_mat(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out)
    exact, mag = oracle.mul_mat_exact(w, x)
    err = oracle.metric(host(out), exact, mag)
    assert err <= oracle.K_B200, f"error {err:.3g}"


@pytest.mark.parametrize("block_n", [128, 256])
def test_mul_mat_config1_bias(cuda, block_n):
    """benchmark config 1: x N(0,1) [4096 x 320], W N(0, 0.02) FP16 [1280 x 320], bias N(0, 0.02)."""
    import sdb

    g = rng(1)
    x = g.standard_normal((4096, 320)).astype(np.float32)
    w = (g.standard_normal((1280, 320)) * 0.02).astype(np.float32).astype(np.float16)
    b = (g.standard_normal(1280) * 0.02).astype(np.float32)
    out = canary_like((4096, 1280), cuda)
    bt = cuda_tensor(b, cuda)
    sdb.set_tuning(f"block_n={block_n}")
    try:
        sdb.mul_mat(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out, chain=sdb.Chain().add(bt))
    finally:
        sdb.set_tuning("block_n=0")
    exact, mag = oracle.mul_mat_exact(w, x)
    exact = exact + b.astype(np.float64)
    mag = mag + np.abs(b.astype(np.float64))
    err = oracle.metric(host(out), exact, mag)
    assert err <= oracle.K_B200, f"error {err:.3g}"


def test_mul_mat_small_and_tiny_rows(cuda):
    """Rows that fill no tile and values far below 1 (the remainder kept normal)."""
    import sdb

    g = rng(7)
    w = oracle.uniform(g, (33, 48), 0.25, np.float16)
    x = (oracle.uniform(g, (5, 48), 1.0) * np.float32(1e-3)).astype(np.float32)
    out = canary_like((5, 33), cuda)
    sdb.mul_mat(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out)
    exact, mag = oracle.mul_mat_exact(w, x)
    assert oracle.metric(host(out), exact, mag) <= oracle.K_B200


# (k, half, m, batch) -- ops_test.cc:946-949
GATED_CASES = [
    (320, 1280, 200, 2),
    (1280, 5120, 64, 2),
    (40, 100, 37, 1),
    (96, 2000, 1500, 1),
]


@pytest.mark.parametrize("k,half,m,batch", GATED_CASES)
def test_gated_gelu_reference_cases(cuda, k, half, m, batch):
    import sdb

    g = rng()
    w = oracle.uniform(g, (2 * half, k), 0.25, np.float16)
    x = oracle.uniform(g, (batch, m, k), 1.0)
    b = oracle.uniform(g, (2 * half,), 1.0)
    out = canary_like((batch, m, half), cuda)
    bt = cuda_tensor(b, cuda)
    sdb.mul_mat_gated(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out, chain=sdb.Chain().add(bt))
    exact, mag = oracle.gated_exact(w, x, b)
    err = oracle.metric(host(out), exact, mag)
    assert err <= oracle.K_B200, f"error {err:.3g}"


def test_fp16_range_flag(cuda):
    """An activation beyond FP16's range is reported in the device error word, not silently wrong."""
    import sdb

    w = np.ones((16, 16), dtype=np.float16)
    x = np.ones((4, 16), dtype=np.float32)
    x[2, 3] = 1e6
    out = canary_like((4, 16), cuda)
    sdb.mul_mat(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out)
    status = sdb.device_status(clear=True)
    assert status & 2, f"range bit not set: 0x{status:x}"


@pytest.mark.parametrize("k", [320, 2560, 11520])
def test_mul_mat_long_sums_of_one_sign(cuda, k):
    """Sums whose products all have one sign, beyond the reference's test
    distributions: the tensor core's accumulation rounds toward zero, so the
    kernel sums each k-block apart (without that, 2.2e-6 at K = 320 and 7.8e-5
    at K = 11520, measured).  What remains is FP32 rounding of the block sums,
    so the bound is 1e-6 or the error of the reference's own form -- an FP32
    running sum over k (mul_mat.cc:306-366) -- on the same outputs, whichever
    is larger."""
    import sdb

    g = rng(11)
    x = g.uniform(0, 1, (256, k)).astype(np.float32)
    w = g.uniform(0, 0.25, (128, k)).astype(np.float16)
    out = canary_like((256, 128), cuda)
    sdb.mul_mat(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out)
    exact, mag = oracle.mul_mat_exact(w, x)
    err = oracle.metric(host(out), exact, mag)
    ref = oracle.mul_mat_f32_running(w, x)
    ref_err = oracle.metric(ref, exact, mag)
    assert err <= max(oracle.K_B200, ref_err), f"error {err:.3g} (reference form {ref_err:.3g})"
