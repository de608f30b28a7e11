"""Parity of attention (FLASH_ATTN_EXT, no mask) against the exact oracle.

Cases: the reference's (tests/ops_test.cc:925-938) -- SD 1.5's self- and
cross-attention made smaller, heads of 80 and 160, the VAE's single head of
512, dims and keys of no multiple of a panel with heads sharing keys, FP16
keys and values -- and benchmark config 3 (8 heads x 40, Lq = Lk = 4096 and
Lk = 77), with and without the residual add fused; heads wider than 160 dims
(the VAE's 512) at full size, with shared FP16 keys and an odd width.  Q, K, V ~ U(-1, 1)
(ops_test.cc:478-483); bound: the ops_test metric <= 1e-6.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

import oracle
from helpers import canary_like, cuda_tensor, host, rng

pytestmark = pytest.mark.gpu

# (d, lq, lk, h, hk, b, kv dtype) -- ops_test.cc:925-938
ATTN_CASES = [
    (40, 300, 4096, 2, 2, 2, np.float32),
    (40, 200, 77, 2, 2, 2, np.float32),
    (80, 100, 1024, 2, 2, 1, np.float32),
    (160, 64, 256, 2, 2, 2, np.float32),
    (512, 40, 300, 1, 1, 1, np.float32),
    (13, 37, 29, 4, 2, 3, np.float32),
    (64, 50, 100, 2, 1, 1, np.float16),
]


def run(cuda, d, lq, lk, h, hk, b, kvtype, seed=oracle.SEED, normal=False, residual=False):
    import sdb

    g = rng(seed)
    if normal:
        q = g.standard_normal((b, lq, h * d)).astype(np.float32)
        k = g.standard_normal((b, lk, hk * d)).astype(np.float32).astype(kvtype)
        v = g.standard_normal((b, lk, hk * d)).astype(np.float32).astype(kvtype)
    else:
        q = oracle.uniform(g, (b, lq, h * d), 1.0)
        k = oracle.uniform(g, (b, lk, hk * d), 1.0, kvtype)
        v = oracle.uniform(g, (b, lk, hk * d), 1.0, kvtype)
    scale = 1.0 / math.sqrt(d)
    out = canary_like((b, lq, h * d), cuda)
    chain = None
    res = None
    if residual:
        res = g.standard_normal((b, lq, h * d)).astype(np.float32)
        rt = cuda_tensor(res, cuda)
        # dst is [DV, H, LQ, B]; the residual [H*DV, LQ, B] seen with the same coordinates.
        chain = sdb.Chain().add(rt, nb=[1, d, h * d, lq * h * d])
    sdb.attention_heads(cuda_tensor(q, cuda), cuda_tensor(k, cuda), cuda_tensor(v, cuda), h, hk, scale, out=out,
                        chain=chain)
    exact, mag = oracle.attention_exact(q, k, v, h, hk, scale)
    if residual:
        exact = exact + res.astype(np.float64)
        mag = mag + np.abs(res.astype(np.float64))
    return oracle.metric(host(out), exact, mag)


@pytest.mark.parametrize("case", ATTN_CASES, ids=lambda c: f"d{c[0]}_q{c[1]}_k{c[2]}_h{c[3]}_{c[4]}_b{c[5]}")
def test_attention_reference_cases(cuda, case):
    import sdb

    err = run(cuda, *case)
    assert err <= oracle.K_B200, f"error {err:.3g}"


@pytest.mark.parametrize("case", [(512, 4096, 4096, 1, 1, 2, np.float32), (256, 77, 130, 3, 1, 2, np.float16),
                                  (200, 33, 64, 2, 2, 1, np.float32)],
                         ids=["vae_512x4096_b2", "d256_shared_kv_f16", "d200"])
def test_attention_wide_heads(cuda, case):
    """Heads over 160 dims (the product, softmax, product path): the SD 1.5 VAE's full-size
    block (one 512-dim head over 4096 positions), heads sharing FP16 keys, an odd width."""
    err = run(cuda, *case)
    assert err <= oracle.K_B200, f"error {err:.3g}"


def test_attention_wide_heads_take_no_chain(cuda):
    import sdb
    import torch

    q = torch.zeros((1, 40, 512), device=cuda)
    out = torch.empty_like(q)
    with pytest.raises(sdb.SdbError, match="take no chain"):
        sdb.attention_heads(q, q, q, 1, 1, 1.0, out=out, chain=sdb.Chain().add(q, nb=[1, 512, 512, 40 * 512]))


@pytest.mark.parametrize("lk,residual", [(4096, False), (77, False), (4096, True), (77, True)])
def test_attention_config3(cuda, lk, residual):
    """benchmark config 3: 8 heads x 40, Lq = 4096, Q/K/V ~ N(0, 1), optional fused residual."""
    err = run(cuda, 40, 4096, lk, 8, 8, 1, np.float32, seed=5, normal=True, residual=residual)
    assert err <= oracle.K_B200, f"error {err:.3g}"


KERNEL_CASES = [c for c in ATTN_CASES if c[0] <= 80] + [(40, 4096, 4096, 8, 8, 1, np.float32),
                                                          (80, 1024, 1024, 8, 8, 2, np.float32)]


@pytest.mark.parametrize("kernel", [2, 1, 0], ids=["tensor_memory_operands", "two_warpgroups", "pairs"])
@pytest.mark.parametrize("case", KERNEL_CASES, ids=lambda c: f"d{c[0]}_q{c[1]}_k{c[2]}_h{c[3]}_{c[4]}_b{c[5]}")
def test_attention_kernels(cuda, case, kernel):
    """Each fused kernel (tuning attention_wg: 2 = two query tiles a CTA, P (and for heads up to 64
    dims Q) in tensor memory; 1 = two softmax warpgroups; 0 = warp pairs) on the reference's cases of
    heads up to 80 dims."""
    import sdb

    before = sdb.get_tuning("attention_wg")
    sdb.set_tuning(f"attention_wg={kernel}")
    try:
        err = run(cuda, *case)
    finally:
        sdb.set_tuning(f"attention_wg={before}")
    assert err <= oracle.K_B200, f"error {err:.3g}"


@pytest.mark.parametrize("lk", [64, 65, 127, 4096])
def test_attention_negative_scale(cuda, lk):
    """A negative scale: the block's largest scaled score is its smallest score (full and ragged key blocks)."""
    import sdb

    g = rng(11)
    d, lq, h, b = 40, 200, 2, 1
    q = oracle.uniform(g, (b, lq, h * d), 1.0)
    k = oracle.uniform(g, (b, lk, h * d), 1.0)
    v = oracle.uniform(g, (b, lk, h * d), 1.0)
    scale = -1.5 / math.sqrt(d)
    out = canary_like((b, lq, h * d), cuda)
    sdb.attention_heads(cuda_tensor(q, cuda), cuda_tensor(k, cuda), cuda_tensor(v, cuda), h, h, scale, out=out)
    exact, mag = oracle.attention_exact(q, k, v, h, h, scale)
    err = oracle.metric(host(out), exact, mag)
    assert err <= oracle.K_B200, f"error {err:.3g}"
