"""Generates the golden fixtures from the reference's own kernels.

    python tests/golden/make_golden.py

Runs in the build container, where the reference's sources are: oracle/
ref_asm.py assembles its x86-64 kernels into oracle/_ref/libsdasm_ref.so and
oracle/ref_driver.c drives them as the reference does.  For each case the
inputs are regenerated from a recorded seed (numpy PCG64, the same on every
machine), so the fixture holds the seed, the shapes and the reference's
outputs only:
  mul_mat   the reference's mul_mat cases with FP16 weights (tests/ops_test.cc:
            825-832), rows cut to keep the fixture small; U(-0.25, 0.25)
            weights, U(-1, 1) inputs (ops_test.cc:441-444)
  gelu      sdasm_gated_gelu_avx2: x GELU(gate) over 1000 pairs
  exp       sdasm_exponentials_avx2: a panel of 64 keys x 16 queries of
            scaled scores, with their per-query maxima and double sums
Writes tests/golden/golden.npz.
"""
from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "oracle"))

MUL_MAT_CASES = [  # (k, n, m) -- ops_test.cc:825-832, rows cut
    (320, 320, 64),
    (768, 1280, 16),
    (1280, 320, 32),
    (300, 17, 31),
]
SEED = 20261011


def inputs_mul_mat(k: int, n: int, m: int, seed: int):
    g = np.random.Generator(np.random.PCG64(seed))
    w = g.uniform(-0.25, 0.25, (n, k)).astype(np.float32).astype(np.float16)
    x = g.uniform(-1.0, 1.0, (m, k)).astype(np.float32)
    return w, x


def inputs_gelu(seed: int):
    g = np.random.Generator(np.random.PCG64(seed))
    x = g.uniform(-4, 4, 1000).astype(np.float32)
    gate = g.uniform(-6, 6, 1000).astype(np.float32)
    return x, gate


def inputs_exp(seed: int):
    g = np.random.Generator(np.random.PCG64(seed))
    s = (g.standard_normal((64, 16)) * 3).astype(np.float32)
    return s, s.max(axis=0).astype(np.float32)


def load_ref():
    import ref_asm

    lib = ctypes.CDLL(str(ref_asm.build()))
    P = ctypes.c_void_p
    lib.refk_mul_mat.argtypes = [P, ctypes.c_int, ctypes.c_int, P, ctypes.c_int, P]
    lib.refk_gated_gelu.argtypes = [P, P, P, ctypes.c_int64]
    lib.refk_exponentials.argtypes = [P, ctypes.c_int64, P, P]
    return lib


def ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def run_mul_mat(lib, w, x):
    y = np.empty((x.shape[0], w.shape[0]), dtype=np.float32)
    assert lib.refk_mul_mat(ptr(w), w.shape[0], w.shape[1], ptr(x), x.shape[0], ptr(y)) == 0
    return y


def run_gelu(lib, x, gate):
    out = np.empty_like(x)
    lib.refk_gated_gelu(ptr(out), ptr(x), ptr(gate), x.size)
    return out


def run_exp(lib, s, mx):
    # The kernel wants its panel 32-byte aligned.
    buf = np.empty(s.size + 16, dtype=np.float32)
    off = (-buf.ctypes.data % 32) // 4
    panel = buf[off:off + s.size].reshape(s.shape)
    panel[...] = s
    total = np.zeros(16, dtype=np.float64)
    lib.refk_exponentials(ptr(panel), s.shape[0], ptr(mx), ptr(total))
    return panel.copy(), total


def main() -> None:
    lib = load_ref()
    out = {}
    for i, (k, n, m) in enumerate(MUL_MAT_CASES):
        w, x = inputs_mul_mat(k, n, m, SEED + i)
        out[f"mul_mat_{i}"] = run_mul_mat(lib, w, x)
    x, gate = inputs_gelu(SEED)
    out["gelu"] = run_gelu(lib, x, gate)
    s, mx = inputs_exp(SEED)
    out["exp"], out["exp_total"] = run_exp(lib, s, mx)
    out["cases"] = np.array(MUL_MAT_CASES, dtype=np.int64)
    out["seed"] = np.array([SEED], dtype=np.int64)
    np.savez_compressed(HERE / "golden.npz", **out)
    print(f"wrote {HERE / 'golden.npz'}")


if __name__ == "__main__":
    main()
