"""The oracle and the kernels against the golden fixtures made by the reference's own kernels.

tests/golden/golden.npz holds outputs of the reference's hand-written x86-64
kernels (sdasm_gemm_6x16_avx2, sdasm_gated_gelu_avx2, sdasm_exponentials_avx2),
assembled from its sources and driven as the reference drives them
(oracle/ref_asm.py, oracle/ref_driver.c, tests/golden/make_golden.py), for
inputs regenerated here from recorded seeds.  The reference judges its forms by
the error relative to the magnitudes against the exact result
(tests/ops_test.cc:157: within 1e-5); its README measures its AVX2 linear
layers at 0.4-2.4e-7.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

import oracle
import ref_asm

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))
import make_golden as mg  # noqa: E402

GOLDEN = np.load(HERE / "golden" / "golden.npz")


def gelu_double(x):
    x = np.asarray(x, dtype=np.float64)
    return 0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


@pytest.mark.parametrize("i", range(len(mg.MUL_MAT_CASES)))
def test_reference_kernels_pin_the_oracle(i):
    """The reference's own GEMM is within its kSingle of the oracle's exact result -- and
    within the precision its README reports (<= 2.4e-7)."""
    k, n, m = mg.MUL_MAT_CASES[i]
    w, x = mg.inputs_mul_mat(k, n, m, mg.SEED + i)
    ex, mag = oracle.mul_mat_exact(w, x)
    err = oracle.metric(GOLDEN[f"mul_mat_{i}"], ex, mag)
    assert err <= 2.4e-7, f"reference kernel vs oracle: {err:.3g}"


def test_reference_gelu_and_oracle_gelu_agree():
    """sdasm_gated_gelu_avx2 and the oracle's restatement of scalar_math.h's GELU are both
    close to the tanh GELU in double (each its own approximation of exp)."""
    x, gate = mg.inputs_gelu(mg.SEED)
    exact = x.astype(np.float64) * gelu_double(gate)
    scale = np.maximum(np.abs(x.astype(np.float64)) * np.abs(gate.astype(np.float64)), 1e-30)
    ref_err = np.max(np.abs(GOLDEN["gelu"] - exact) / scale)
    ora_err = np.max(np.abs(x * oracle.gelu(gate) - exact) / scale)
    assert ref_err < 2e-6 and ora_err < 2e-6, (ref_err, ora_err)


def test_reference_exponentials_and_sums():
    """sdasm_exponentials_avx2's exponentials and double sums against the double
    exponential; the oracle's exponential() (scalar_math.h) against the same."""
    s, mx = mg.inputs_exp(mg.SEED)
    arg = (s - mx).astype(np.float32).astype(np.float64)  # the kernels' FP32 argument
    e = np.exp(arg)
    assert np.max(np.abs(GOLDEN["exp"] - e) / e) < 4e-7
    assert np.max(np.abs(GOLDEN["exp_total"] - e.sum(axis=0)) / e.sum(axis=0)) < 1e-7
    assert np.max(np.abs(oracle.exponential((s - mx).astype(np.float32)) - e) / e) < 4e-7


def test_fixture_reproduces_from_the_reference():
    """Regenerated from the reference's kernels (where its sources are), the fixture is bit-identical."""
    if not ref_asm.reference_kernels_present():
        pytest.skip("the reference's sources are not on this machine")
    lib = mg.load_ref()
    for i, (k, n, m) in enumerate(mg.MUL_MAT_CASES):
        w, x = mg.inputs_mul_mat(k, n, m, mg.SEED + i)
        assert np.array_equal(mg.run_mul_mat(lib, w, x), GOLDEN[f"mul_mat_{i}"])


@pytest.mark.gpu
@pytest.mark.parametrize("i", range(len(mg.MUL_MAT_CASES)))
def test_kernels_match_the_reference_kernels(cuda, i):
    """The B200 linear layer on the fixture's inputs: within 1e-6 of the exact result, and
    within 1e-6 (relative to the magnitudes) of the reference's own kernel's output."""
    import sdb
    import torch

    k, n, m = mg.MUL_MAT_CASES[i]
    w, x = mg.inputs_mul_mat(k, n, m, mg.SEED + i)
    out = sdb.mul_mat(torch.from_numpy(w).to(cuda), torch.from_numpy(x).to(cuda)).cpu().numpy()
    ex, mag = oracle.mul_mat_exact(w, x)
    assert oracle.metric(out, ex, mag) <= oracle.K_B200
    ref = GOLDEN[f"mul_mat_{i}"].astype(np.float64)
    assert oracle.metric(out, ref, mag) <= 1e-6
