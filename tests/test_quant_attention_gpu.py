"""Parity of attention with integer products (tuning bits = 2..8, quantize's attention bit).

The reference quantizes self-attention over 256 keys and more and leaves attention
over fewer (the prompt's 77 tokens) in single precision (attention.cc:612-618).
The cases are its quantized attention cases (ops_test.cc:905-916) and its narrower
integers (ops_test.cc:903-904).

Bounds, as the reference holds its own quantized attention forms to them
(ops_test.cc:213-239): within kQuantized (1e-2 with 8 bits of both operands, in
proportion to 2/L + 1/W with fewer) of the exact attention, and within
kQuantizedApart (1e-3) of the reference's C++ form (oracle/ref_forms.py
qattention), relative to the magnitudes -- not bit for bit: an exponential that
differs from the form's in its last bit (the GPU's expf for the keys past the
last eight, or a double sum in another order) can round to the next step of 8
bits, a step of a group of keys.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

import oracle
import ref_forms
from helpers import canary_like, cuda_tensor, host, rng
from test_quant_gpu import bound, tuned

pytestmark = pytest.mark.gpu

APART = 1e-3

# (d, lq, lk, h, hk, b, kv dtype): ops_test.cc:905-916 with lk >= 256.
CASES = [
    (40, 300, 4096, 2, 2, 2, np.float32),
    (80, 100, 1024, 2, 2, 1, np.float16),
    (160, 64, 256, 2, 2, 2, np.float32),
    (13, 37, 290, 4, 2, 3, np.float32),
]


def ids(c):
    return f"d{c[0]}_q{c[1]}_k{c[2]}_h{c[3]}_{c[4]}_b{c[5]}_{np.dtype(c[6]).name}"


def run(cuda, d, lq, lk, h, hk, b, kvtype, seed=oracle.SEED, residual=None):
    import sdb

    g = rng(seed)
    q = oracle.uniform(g, (b, lq, h * d), 1.0)
    k = oracle.uniform(g, (b, lk, hk * d), 1.0, kvtype)
    v = oracle.uniform(g, (b, lk, hk * d), 1.0, kvtype)
    scale = 1.0 / math.sqrt(d)
    out = canary_like((b, lq, h * d), cuda)
    chain = None
    if residual is not None:
        chain = sdb.Chain().add(cuda_tensor(residual, cuda), nb=[1, d, h * d, lq * h * d])
    sdb.attention_heads(cuda_tensor(q, cuda), cuda_tensor(k, cuda), cuda_tensor(v, cuda), h, hk, scale, out=out,
                        chain=chain)
    return q, k, v, scale, host(out)


def check(got, q, k, v, h, hk, scale, group=64, bits=8, input_bits=8, extra=None):
    form = ref_forms.qattention(q, k, v, h, hk, scale, group, (1 << input_bits) - 1, (1 << (bits - 1)) - 1)
    exact, mag = oracle.attention_exact(q, k, v, h, hk, scale)
    if extra is not None:
        form = form + extra
        exact = exact + extra.astype(np.float64)
        mag = mag + np.abs(extra.astype(np.float64))
    apart = oracle.metric(got, form, mag)
    err = oracle.metric(got, exact, mag)
    assert apart <= APART, f"{apart:.3g} from the C++ form"
    assert err <= bound(bits, input_bits), f"error {err:.3g}"


@pytest.mark.parametrize("case", CASES, ids=ids)
def test_quantized_attention_reference_cases(cuda, case):
    d, lq, lk, h, hk, b, kvtype = case
    with tuned("bits=8"):
        q, k, v, scale, got = run(cuda, *case)
    check(got, q, k, v, h, hk, scale)


@pytest.mark.parametrize("bits,input_bits", [(7, 8), (8, 7)])
@pytest.mark.parametrize("case", [CASES[0], CASES[3]], ids=ids)
def test_quantized_attention_narrow_integers(cuda, case, bits, input_bits):
    d, lq, lk, h, hk, b, kvtype = case
    with tuned(f"bits={bits},input_bits={input_bits}"):
        q, k, v, scale, got = run(cuda, *case)
    check(got, q, k, v, h, hk, scale, bits=bits, input_bits=input_bits)


@pytest.mark.parametrize("group", [32, 128])
def test_quantized_attention_groups(cuda, group):
    case = CASES[1]
    d, lq, lk, h, hk, b, kvtype = case
    with tuned(f"bits=8,group={group}"):
        q, k, v, scale, got = run(cuda, *case)
    check(got, q, k, v, h, hk, scale, group=group)


def test_quantized_attention_residual(cuda):
    """The chain after the quantized attention (an extension: the UNet runner's residual add)."""
    case = CASES[0]
    d, lq, lk, h, hk, b, kvtype = case
    res = rng(51).standard_normal((b, lq, h * d)).astype(np.float32)
    with tuned("bits=8"):
        q, k, v, scale, got = run(cuda, *case, residual=res)
    check(got, q, k, v, h, hk, scale, extra=res)


def test_few_keys_stay_single_precision(cuda):
    """Cross-attention over 77 keys is not quantized (attention.cc:612-618): the FP32 path's bound."""
    with tuned("bits=8"):
        q, k, v, scale, got = run(cuda, 40, 200, 77, 2, 2, 2, np.float32)
    exact, mag = oracle.attention_exact(q, k, v, 2, 2, scale)
    assert oracle.metric(got, exact, mag) <= oracle.K_B200
