"""The quantized forms (bits = 8) against fixtures made by the reference's own kernels.

tests/golden/golden_quant.npz (tests/golden/make_golden.py) holds, for seeded
inputs, the outputs of two of the reference's hand-written x86-64 kernels,
assembled from its sources (oracle/ref_asm.py):
  sdasm_quantize16_avx2       its quantization of inputs (unsigned, zero point,
                              a scale and offset per group), quant.cc:380-430
  sdasm_qgemm_6x16_au_avx512  its integer sums and per-group fold over quant.h
                              panels, quant.cc:113-166's order
The oracle (oracle/ref_forms.c) reproduces both bit for bit, and the B200
quantized linear layer reproduces the reference kernel's products bit for
bit.  The weights' quantization (quant.cc:204-244) has no hand-written form:
the oracle restates it, and the fixture's products are taken over weights it
quantized.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

import ref_asm
import ref_forms

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE / "golden"))
import make_golden as mg  # noqa: E402

GOLDEN = np.load(HERE / "golden" / "golden_quant.npz")
CASES = [tuple(int(v) for v in c) for c in GOLDEN["cases"]]


def columns_panel(q, s, o, group):
    """Quantized rows (16 of them) as the bytes of quant.h's panel of 16 columns."""
    return mg.b_panels(q.view(np.int8), s, o, group)[0].view(np.uint8)


@pytest.mark.parametrize("i", range(len(CASES)))
def test_reference_quantization_pins_the_oracle(i):
    k, n, m, group = CASES[i]
    _, x = mg.inputs_quant(k, n, m, int(GOLDEN["seed"][0]) + i)
    q, s, o = ref_forms.quantize_inputs(x[:16], group)
    assert np.array_equal(columns_panel(q, s, o, group), GOLDEN[f"q16_{i}"])


@pytest.mark.parametrize("i", range(len(CASES)))
def test_reference_product_pins_the_oracle(i):
    k, n, m, group = CASES[i]
    w, x = mg.inputs_quant(k, n, m, int(GOLDEN["seed"][0]) + i)
    y = ref_forms.qmul_mat(w, x[:m], group=group)
    assert np.array_equal(y.view(np.uint32), GOLDEN[f"qmm_{i}"].view(np.uint32))


def test_reference_product_accumulating_pins_the_oracle():
    k, n, m, group = CASES[0]
    w, x = mg.inputs_quant(k, n, m, int(GOLDEN["seed"][0]))
    y = ref_forms.qmul_mat(w, x[:m], group=group, y0=GOLDEN["qmm_acc_y0"])
    assert np.array_equal(y.view(np.uint32), GOLDEN["qmm_acc"].view(np.uint32))


def test_quant_fixture_reproduces_from_the_reference():
    if not ref_asm.reference_kernels_present() or not mg.has_vnni512():
        pytest.skip("the reference's sources or AVX512-VNNI are not on this machine")
    lib = mg.load_ref()
    for i, (k, n, m, group) in enumerate(CASES):
        w, x = mg.inputs_quant(k, n, m, int(GOLDEN["seed"][0]) + i)
        assert np.array_equal(mg.run_quantize16(lib, x[:16], group), GOLDEN[f"q16_{i}"])
        assert np.array_equal(mg.run_qgemm(lib, w, x[:m], group), GOLDEN[f"qmm_{i}"])


@pytest.mark.gpu
@pytest.mark.parametrize("i", range(len(CASES)))
def test_kernel_matches_the_reference_kernel(cuda, i):
    """The B200 quantized product on the fixture's inputs, its rows repeated to the 256 a
    quantized product needs: the reference kernel's outputs, bit for bit."""
    import sdb
    import torch

    k, n, m, group = CASES[i]
    w, x = mg.inputs_quant(k, n, m, int(GOLDEN["seed"][0]) + i)
    rows = np.tile(x[:m], (-(-256 // m), 1))
    sdb.set_tuning(f"bits=8,group={group}")
    try:
        out = sdb.mul_mat(torch.from_numpy(w).to(cuda), torch.from_numpy(rows).to(cuda)).cpu().numpy()
    finally:
        sdb.set_tuning("bits=0,group=64")
    ref = GOLDEN[f"qmm_{i}"]
    for r0 in range(0, rows.shape[0] - m + 1, m):
        assert np.array_equal(out[r0:r0 + m].view(np.uint32), ref.view(np.uint32))
