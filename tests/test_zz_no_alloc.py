"""sdb_group_norm_no_alloc, the GroupNorm that allocates no device memory, against sdb_group_norm.

Collected last (file name) so that it runs both after the other tests and, with
`pytest tests/test_zz_no_alloc.py`, alone in a fresh process.  Each case makes
two calls in a row through the C ABI with different inputs (the second call
finds the first call's partial sums in the shared static array) and holds both
to the GroupNorm tests' bound: within 1e-6 of the largest output of
sdb_group_norm on the same input.
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


def inputs(shape, seed, cuda):
    import sdb

    g = rng(seed)
    x = oracle.uniform(g, shape, 3.0) + np.float32(seed % 5)
    c = shape[1]
    gamma = cuda_tensor(oracle.uniform(g, (1, c, 1, 1), 1.0), cuda)
    beta = cuda_tensor(oracle.uniform(g, (1, c, 1, 1), 1.0), cuda)
    return cuda_tensor(x, cuda), sdb.Chain().mul(gamma).add(beta).silu()


@pytest.mark.parametrize("first,second,groups", [
    ((2, 64, 20, 36), (1, 30, 7, 13), 32),       # ops_test.cc:1083-1106 shapes, one slice per group
    ((1, 320, 64, 64), (1, 1280, 8, 8), 32),     # the UNet's GroupNorms (several slices per group)
    ((1, 512, 64, 64), (2, 512, 64, 64), 32),    # VAE-sized groups (the split path of both entry points)
])
def test_no_alloc_matches_group_norm_twice(cuda, first, second, groups):
    import sdb
    import torch

    for call, shape in enumerate((first, second)):
        x, chain = inputs(shape, oracle.SEED + call, cuda)
        got = canary_like(shape, cuda)
        want = canary_like(shape, cuda)
        sdb.group_norm_no_alloc(x, groups, 1e-5, out=got, chain=chain)
        sdb.group_norm(x, groups, 1e-5, out=want, chain=chain)
        torch.cuda.synchronize()
        close(host(got), host(want))


def test_no_alloc_repeat_allocates_nothing(cuda):
    """After the first call on the device, a call changes the device's free memory by nothing."""
    import sdb
    import torch

    x, chain = inputs((1, 640, 32, 32), oracle.SEED, cuda)
    out = canary_like(x.shape, cuda)
    sdb.group_norm_no_alloc(x, 32, 1e-5, out=out, chain=chain)
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info()
    for _ in range(2):
        sdb.group_norm_no_alloc(x, 32, 1e-5, out=out, chain=chain)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before


def test_no_alloc_rejects_sizes_beyond_its_scratch(cuda):
    import sdb

    x = cuda_tensor(np.zeros((3, 16384, 1, 1), dtype=np.float32), cuda)   # 3 x 16384 groups > 32768
    out = canary_like(x.shape, cuda)
    with pytest.raises(sdb.SdbError, match="exceeds the static scratch limit"):
        sdb.group_norm_no_alloc(x, 16384, 1e-5, out=out)
