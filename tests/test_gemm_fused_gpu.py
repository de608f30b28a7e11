"""The linear layers' GEMM that splits its FP32 activations itself (gemm_fused.cuh).

It reads x as FP32 rows by TMA, splits them in shared memory into the FP16
pairs of tensor memory's A operand, and sums a k-block's hi and lo products in
one accumulator.  These cases (gemm_fused=2: the fused kernel for every
product it can take) reach each tile width (128, 160, 192), the K split with
its reduction, gated products at each width, rows and K that fill no tile, and
the pre-pass path it replaces (gemm_fused=0, and x whose rows TMA cannot
tile); every result is held to the ops_test metric against float64 (<= 1e-6),
as the reference's MUL_MAT cases are.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from helpers import canary_like, cuda_tensor, host, rng

pytestmark = pytest.mark.gpu


class tuned:
    def __init__(self, spec):
        self.spec = spec

    def __enter__(self):
        import sdb

        sdb.set_tuning(self.spec)

    def __exit__(self, *exc):
        import sdb

        sdb.set_tuning("block_n=0,gemm_fused=1")


# (k, n, rows, block_n): widths forced, rows past a tile, K not a multiple of 64
CASES = [
    (320, 320, 1000, 160),
    (320, 320, 1000, 192),
    (320, 320, 1000, 128),
    (640, 640, 4096, 0),
    (100, 96, 77, 0),          # K = 100: the last k-block half outside the rows (TMA's zero fill)
    (36, 50, 5, 0),
    (2560, 320, 256, 0),       # few tiles, long K: split over CTAs, then the reduction
    (1280, 1280, 300, 0),
    (5120, 1280, 200, 0),
]


@pytest.mark.parametrize("k,n,rows,block_n", CASES)
def test_fused_linear_bias_residual(cuda, k, n, rows, block_n):
    import sdb

    g = rng(k + n + rows)
    w = oracle.uniform(g, (n, k), 0.25, np.float16)
    x = oracle.uniform(g, (rows, k), 1.0)
    b = oracle.uniform(g, (n,), 1.0)
    r = oracle.uniform(g, (rows, n), 1.0)
    out = canary_like((rows, n), cuda)
    with tuned(f"block_n={block_n},gemm_fused=2"):
        sdb.mul_mat(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out,
                    chain=sdb.Chain().add(cuda_tensor(b, cuda)).add(cuda_tensor(r, cuda)))
    assert sdb.device_status(clear=True) == 0
    exact, mag = oracle.mul_mat_exact(w, x)
    exact = exact + b.astype(np.float64) + r.astype(np.float64)
    mag = mag + np.abs(b.astype(np.float64)) + np.abs(r.astype(np.float64))
    err = oracle.metric(host(out), exact, mag)
    assert err <= oracle.K_B200, f"error {err:.3g}"


@pytest.mark.parametrize("block_n", [128, 160, 192])
@pytest.mark.parametrize("k,half,rows", [(320, 1280, 700), (640, 200, 130)])
def test_fused_gated(cuda, k, half, rows, block_n):
    import sdb

    g = rng(half + rows)
    w = oracle.uniform(g, (2 * half, k), 0.25, np.float16)
    x = oracle.uniform(g, (rows, k), 1.0)
    b = oracle.uniform(g, (2 * half,), 1.0)
    out = canary_like((rows, half), cuda)
    with tuned(f"block_n={block_n},gemm_fused=2"):
        sdb.mul_mat_gated(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out, chain=sdb.Chain().add(cuda_tensor(b, cuda)))
    assert sdb.device_status(clear=True) == 0
    exact, mag = oracle.gated_exact(w, x, b)
    err = oracle.metric(host(out), exact, mag)
    assert err <= oracle.K_B200, f"error {err:.3g}"


@pytest.mark.parametrize("fused", [0, 2])
def test_fused_and_prepass_one_sign(cuda, fused):
    """Both paths of the linear layers stay within the bound on the UNet's most frequent shape
    (two images' 4096 tokens x 320 channels) with one-sign sums."""
    import sdb

    g = rng(5)
    x = g.uniform(0, 1, (8192, 320)).astype(np.float32)
    w = g.uniform(0, 0.25, (320, 320)).astype(np.float16)
    out = canary_like((8192, 320), cuda)
    with tuned(f"gemm_fused={fused}"):
        sdb.mul_mat(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out)
    exact, mag = oracle.mul_mat_exact(w, x)
    err = oracle.metric(host(out), exact, mag)
    assert err <= oracle.K_B200, f"error {err:.3g}"


def test_rows_tma_cannot_tile_take_the_prepass(cuda):
    """K % 4 != 0 (a row pitch TMA cannot take): the pre-pass path, same bound."""
    import sdb

    g = rng(9)
    w = oracle.uniform(g, (64, 77), 0.25, np.float16)
    x = oracle.uniform(g, (2, 50, 77), 1.0)
    out = canary_like((2, 50, 64), cuda)
    with tuned("gemm_fused=2"):
        sdb.mul_mat(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out)
    exact, mag = oracle.mul_mat_exact(w, x)
    assert oracle.metric(host(out), exact, mag) <= oracle.K_B200


def test_fp16_range_flag_fused(cuda):
    """An activation beyond FP16's range sets the device error word on the fused path too."""
    import sdb

    w = np.ones((16, 16), dtype=np.float16)
    x = np.ones((4, 16), dtype=np.float32)
    x[2, 3] = 1e6
    out = canary_like((4, 16), cuda)
    with tuned("gemm_fused=2"):
        sdb.mul_mat(cuda_tensor(w, cuda), cuda_tensor(x, cuda), out)
    status = sdb.device_status(clear=True)
    assert status & 2, f"range bit not set: 0x{status:x}"
