"""Group and layer normalisation with their chains against the reference's algorithm.

The reference's own check of these is fused-vs-apart within 1e-6 of the
largest output (ops_test.cc:1083-1117): GN of [36, 20, 64, 2] in 32 groups,
eps 1e-6, then scale, shift, SiLU; GN of [13, 7, 30, 1] in 10 groups, eps
1e-5; LN of [320, 77, 2], eps 1e-5, then scale and shift.  Here the GPU
result is held to within 1e-6 of the largest output of the reference's
algorithm restated on the CPU (oracle.group_norm_ref / norm_ref, norm.cc),
with the chain applied apart (oracle.apply_chain, fusion.cc:77-86).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from helpers import canary_like, cuda_tensor, host, rng

pytestmark = pytest.mark.gpu


def close(got, want, bound=oracle.K_FUSED_APART):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert np.all(np.isfinite(got)), "non-finite output (canary left?)"
    largest = np.abs(want).max()
    diff = np.abs(got - want).max()
    assert diff <= bound * largest, f"{diff / largest:.3g} of the largest output"


@pytest.mark.parametrize("shape,groups,eps,silu", [
    ((2, 64, 20, 36), 32, 1e-6, True),     # ops_test.cc:1083-1094
    ((1, 30, 7, 13), 10, 1e-5, True),      # ops_test.cc:1095-1106 (rows of no multiple of eight)
    ((1, 320, 64, 64), 32, 1e-5, True),    # benchmark config 2a's GroupNorm
    ((1, 1280, 8, 8), 32, 1e-5, True),     # config 2c
])
def test_group_norm_chain(cuda, shape, groups, eps, silu):
    import sdb

    g = rng()
    x = oracle.uniform(g, shape, 3.0)
    c = shape[1]
    gamma = oracle.uniform(g, (1, c, 1, 1), 1.0)
    beta = oracle.uniform(g, (1, c, 1, 1), 1.0)
    gt, bt = cuda_tensor(gamma, cuda), cuda_tensor(beta, cuda)
    chain = sdb.Chain().mul(gt).add(bt)
    steps = [("mul", gamma), ("add", beta)]
    if silu:
        chain.silu()
        steps.append(("silu", None))
    out = canary_like(shape, cuda)
    sdb.group_norm(cuda_tensor(x, cuda), groups, eps, out=out, chain=chain)
    want = oracle.apply_chain(oracle.group_norm_ref(x, groups, eps), steps)
    close(host(out), want)


def test_layer_norm_chain(cuda):
    """ops_test.cc:1107-1117: LN of [320, 77, 2], eps 1e-5, then scale and shift."""
    import sdb

    g = rng()
    x = oracle.uniform(g, (2, 77, 320), 3.0)
    gamma = oracle.uniform(g, (320,), 1.0)
    beta = oracle.uniform(g, (320,), 1.0)
    out = canary_like(x.shape, cuda)
    chain = sdb.Chain().mul(cuda_tensor(gamma, cuda)).add(cuda_tensor(beta, cuda))
    sdb.norm(cuda_tensor(x, cuda), 1e-5, out=out, chain=chain)
    want = oracle.apply_chain(oracle.norm_ref(x, 1e-5), [("mul", gamma), ("add", beta)])
    close(host(out), want)


@pytest.mark.parametrize("shape", [
    (1, 77, 320),    # two rows a warp, an odd row count (the last warp's second row empty)
    (3, 5, 256),     # 15 rows of 256 (eight numbers a lane)
    (2, 9, 384),     # rows of 384: the widest of the two-rows-a-warp form
    (1, 7, 640),     # one row a warp, 20 numbers a lane
    (1, 3, 1280),    # 40 numbers a lane
    (1, 5, 200),     # a row that ends inside a lane's numbers
    (1, 2, 1500),    # wider than the register forms: the shared-memory kernel
])
def test_layer_norm_row_forms(cuda, shape):
    """Every LayerNorm row form against the oracle, with a canary output and a gamma/beta chain."""
    import sdb

    g = rng(sum(shape))
    x = oracle.uniform(g, shape, 3.0) + np.float32(0.5)
    c = shape[-1]
    gamma = oracle.uniform(g, (c,), 1.0)
    beta = oracle.uniform(g, (c,), 1.0)
    out = canary_like(x.shape, cuda)
    chain = sdb.Chain().mul(cuda_tensor(gamma, cuda)).add(cuda_tensor(beta, cuda))
    sdb.norm(cuda_tensor(x, cuda), 1e-5, out=out, chain=chain)
    want = oracle.apply_chain(oracle.norm_ref(x, 1e-5), [("mul", gamma), ("add", beta)])
    close(host(out), want)


def test_group_norm_matches_double(cuda):
    """The statistics in double: the result is within FP32 rounding of the exact normalisation."""
    import sdb

    g = rng(3)
    x = (g.standard_normal((1, 640, 32, 32)) * 4 + 1).astype(np.float32)
    out = sdb.group_norm(cuda_tensor(x, cuda), 32, 1e-5)
    exact = oracle.group_norm_exact(x, 32, 1e-5)
    assert np.abs(host(out) - exact).max() <= 2e-6 * np.abs(exact).max()


@pytest.mark.parametrize("shape,groups", [
    ((2, 64, 64, 320), 32),    # the UNet's first level, CFG batch 2
    ((2, 32, 32, 640), 32),
    ((1, 8, 8, 1280), 32),
    ((2, 16, 16, 2560), 32),   # decoder concatenations
    ((1, 5, 7, 96), 8),        # ragged positions
])
def test_group_norm_channels_last(cuda, shape, groups):
    """Channels-last images (N, H, W, C): the same algorithm, the same bound."""
    import sdb

    g = rng(11)
    n, h, w, c = shape
    x = oracle.uniform(g, shape, 3.0) + np.float32(0.5)
    gamma = oracle.uniform(g, (c,), 1.0)
    beta = oracle.uniform(g, (c,), 1.0)
    chain = sdb.Chain().mul(cuda_tensor(gamma, cuda), [0, 0, 1, 0]).add(cuda_tensor(beta, cuda), [0, 0, 1, 0]).silu()
    out = canary_like(shape, cuda)
    sdb.group_norm_nhwc(cuda_tensor(x, cuda), groups, 1e-5, out=out, chain=chain)
    nchw = np.ascontiguousarray(x.transpose(0, 3, 1, 2))
    want = oracle.apply_chain(oracle.group_norm_ref(nchw, groups, 1e-5),
                              [("mul", gamma.reshape(1, c, 1, 1)), ("add", beta.reshape(1, c, 1, 1)), ("silu", None)])
    close(host(out).transpose(0, 3, 1, 2), want)
