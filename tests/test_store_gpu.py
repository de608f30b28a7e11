"""The weight store: packed weights are reused, and forgotten when their memory changes.

The reference's test (ops_test.cc:643-719): compute, set the weights anew
through ggml (which calls sdasm_forget), compute again -- the output must be
a fresh computation's (within 1e-6 of the largest) and must have moved from
the old one (by more than 1e-3 of the largest).  Here the weights are
rewritten in place and sdb_forget is called, as ggml's patched buffer writes
do; the cases are the reference's five (conv2d, conv2d by Winograd, conv2d of
shared columns, linear, linear of shared rows).
"""
from __future__ import annotations

import numpy as np
import pytest

from helpers import cuda_tensor, host, rng

pytestmark = pytest.mark.gpu


def _conv(wshape, xshape):
    def run(sdb, w, x):
        return sdb.conv2d(w, x, (1, 1), (1, 1), (1, 1))
    return wshape, xshape, run


def _linear(wshape, xshape):
    def run(sdb, w, x):
        return sdb.mul_mat(w, x)
    return wshape, xshape, run


CASES = {
    "conv2d": _conv((24, 16, 3, 3), (2, 16, 12, 20)),
    "conv2d by Winograd": _conv((24, 16, 3, 3), (1, 16, 32, 64)),
    "conv2d of shared columns": _conv((64, 40, 3, 3), (2, 40, 8, 8)),
    "linear": _linear((80, 64), (2000, 64)),
    "linear of shared rows": _linear((80, 64), (50, 64)),
}


@pytest.mark.parametrize("name", list(CASES))
def test_store_forget(cuda, name):
    import sdb
    import torch

    wshape, xshape, run = CASES[name]
    g = rng(100)
    x = cuda_tensor(g.uniform(-1, 1, xshape).astype(np.float32), cuda)
    w1 = g.uniform(-1, 1, wshape).astype(np.float16)
    w2 = np.random.default_rng(2).uniform(-1, 1, wshape).astype(np.float16)
    w = cuda_tensor(w1, cuda)
    old = host(run(sdb, w, x))
    w.copy_(torch.from_numpy(w2).to(cuda))      # set anew, in place
    sdb.forget(w)                               # as ggml's buffer write does
    changed = host(run(sdb, w, x))
    fresh = host(run(sdb, cuda_tensor(w2, cuda), x))
    largest = np.abs(fresh).max()
    assert np.abs(changed - fresh).max() <= 1e-6 * largest, "differs from a fresh computation"
    assert np.abs(changed - old).max() > 1e-3 * largest, "the old packing was kept"


def test_store_reuses_packed_weights(cuda):
    """A second call with the same weights packs nothing: one launch, the
    product (which splits its FP32 activations itself), without the packing;
    with the split pre-pass (gemm_fused=0) two."""
    import sdb

    g = rng(4)
    w = cuda_tensor(g.uniform(-1, 1, (96, 64)).astype(np.float16), cuda)
    x = cuda_tensor(g.uniform(-1, 1, (128, 64)).astype(np.float32), cuda)
    sdb.mul_mat(w, x)
    n0 = sdb.launch_count()
    sdb.mul_mat(w, x)
    assert sdb.launch_count() - n0 == 1
    sdb.set_tuning("gemm_fused=0")
    try:
        n0 = sdb.launch_count()
        sdb.mul_mat(w, x)
        assert sdb.launch_count() - n0 == 2
    finally:
        sdb.set_tuning("gemm_fused=1")
    entries, nbytes = sdb.store_stats()
    assert entries >= 1 and nbytes > 0


def test_store_off_repacks(cuda):
    """With store=0 every call packs anew (pack, product) and keeps nothing."""
    import sdb

    g = rng(5)
    w = cuda_tensor(g.uniform(-1, 1, (96, 64)).astype(np.float16), cuda)
    x = cuda_tensor(g.uniform(-1, 1, (128, 64)).astype(np.float32), cuda)
    sdb.set_tuning("store=0")
    try:
        before = sdb.store_stats()[0]
        n0 = sdb.launch_count()
        a = host(sdb.mul_mat(w, x))
        assert sdb.launch_count() - n0 == 2
        assert sdb.store_stats()[0] <= before
    finally:
        sdb.set_tuning("store=1")
    b = host(sdb.mul_mat(w, x))
    assert np.array_equal(a, b)
