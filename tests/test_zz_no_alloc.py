"""sdb_group_norm_no_alloc, the GroupNorm that allocates no device memory.

Some callers cannot allocate device memory: a host whose device memory is owned
by another allocator, work recorded under stream capture, a loop that must not
take the driver's allocation lock.  The entry point serves them with a fixed
static scratch array; these tests check it against sdb_group_norm (the entry
point that does allocate) and against the float64-summed CPU restatement of the
reference's GroupNorm (oracle.group_norm_ref, norm.cc:100-140).

Collected last (file name) so that it runs both after the other tests and, with
`pytest tests/test_zz_no_alloc.py`, alone in a fresh process.  Each case makes
two calls in a row through the C ABI with different inputs (the second call
finds the first call's partial sums in the shared static array) and holds both
to the GroupNorm tests' bound: within 1e-6 of the largest output, against
sdb_group_norm on the same input and against the oracle.
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
    """x on the device, its chain (scale, shift, SiLU), and what the oracle makes of them."""
    import sdb

    g = rng(seed)
    x = oracle.uniform(g, shape, 3.0) + np.float32(seed % 5)
    c = shape[1]
    gamma = oracle.uniform(g, (1, c, 1, 1), 1.0)
    beta = oracle.uniform(g, (1, c, 1, 1), 1.0)
    chain = sdb.Chain().mul(cuda_tensor(gamma, cuda)).add(cuda_tensor(beta, cuda)).silu()
    return cuda_tensor(x, cuda), chain, (x, [("mul", gamma), ("add", beta), ("silu", None)])


def oracle_group_norm(host_inputs, groups, eps=1e-5):
    x, steps = host_inputs
    return oracle.apply_chain(oracle.group_norm_ref(x, groups, eps), steps)


@pytest.mark.parametrize("first,second,groups", [
    ((2, 64, 20, 36), (1, 30, 7, 13), 32),       # ops_test.cc:1083-1106 shapes, one slice per group
    ((1, 320, 64, 64), (1, 1280, 8, 8), 32),     # the UNet's GroupNorms (several slices per group)
    ((1, 512, 64, 64), (2, 512, 64, 64), 32),    # VAE-sized groups (the split path of both entry points)
])
def test_no_alloc_matches_group_norm_twice(cuda, first, second, groups):
    import sdb
    import torch

    for call, shape in enumerate((first, second)):
        x, chain, on_host = inputs(shape, oracle.SEED + call, cuda)
        got = canary_like(shape, cuda)
        want = canary_like(shape, cuda)
        sdb.group_norm_no_alloc(x, groups, 1e-5, out=got, chain=chain)
        sdb.group_norm(x, groups, 1e-5, out=want, chain=chain)
        torch.cuda.synchronize()
        close(host(got), host(want))
        if np.prod(shape) <= (1 << 21):   # the oracle's Python loop over groups stays in seconds
            close(host(got), oracle_group_norm(on_host, groups))


def test_no_alloc_repeat_allocates_nothing(cuda):
    """After the first call on the device, a call changes the device's free memory by nothing."""
    import sdb
    import torch

    x, chain, _ = inputs((1, 640, 32, 32), oracle.SEED, cuda)
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


def test_no_alloc_rejects_channels_last_images(cuda):
    """Only the contiguous (channel-major) layout is taken; sdb_group_norm also takes channels-last."""
    import sdb
    import torch

    x = torch.zeros((1, 64, 8, 8), dtype=torch.float32, device=cuda).to(memory_format=torch.channels_last)
    out = torch.empty_like(x)
    with pytest.raises(sdb.SdbError, match="not supported"):
        sdb.group_norm_no_alloc(x, 32, 1e-5, out=out)
