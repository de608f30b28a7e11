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
Writes tests/golden/golden.npz, and tests/golden/golden_quant.npz with the
quantized forms (bits = 8; quant.h), where the host has AVX512-VNNI:
  q16       sdasm_quantize16_avx2: the first 16 rows of the inputs quantized
            as a panel of 16 columns (bytes [quads][16][4], 16 scales, 16
            offsets a group) -- the reference's quantization of inputs
  qmm       sdasm_qgemm_6x16_au_avx512 over panels of the inputs and weights
            quantized by oracle/ref_forms.c (laid out as quant.h lays them):
            the reference's integer sums and per-group fold
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


QUANT_CASES = [  # (k, n, m, group): rows a multiple of 6, columns of 16, k of the group
    (320, 64, 24, 64),
    (640, 32, 18, 32),
    (640, 48, 18, 128),
    (1280, 16, 6, 256),
    (768, 32, 24, 64),
]
QUANT_SEED = 20261201


def inputs_quant(k: int, n: int, m: int, seed: int):
    g = np.random.Generator(np.random.PCG64(seed))
    w = g.uniform(-0.25, 0.25, (n, k)).astype(np.float32).astype(np.float16)
    x = g.uniform(-1.0, 1.0, (max(m, 16), k)).astype(np.float32)
    return w, x


def a_panels(q, s, o, group):
    """Quantized rows as quant.h's A panels of 6 rows (Qlayout::rows): per group the
    6 rows' bytes, then 6 scales, then 6 offsets."""
    m, groups = s.shape
    panels = []
    for r0 in range(0, m, 6):
        parts = []
        for gi in range(groups):
            parts.append(q[r0:r0 + 6, gi * group:(gi + 1) * group].reshape(-1).view(np.uint8))
            parts.append(s[r0:r0 + 6, gi].astype(np.float32).view(np.uint8))
            parts.append(o[r0:r0 + 6, gi].astype(np.float32).view(np.uint8))
        panels.append(np.concatenate(parts))
    return panels


def b_panels(q, s, o, group):
    """Quantized weights as quant.h's B panels of 16 columns (Qlayout::columns): per
    group the bytes [quads][16][4], then 16 scales, then 16 offsets."""
    n, groups = s.shape
    quads = group // 4
    panels = []
    for c0 in range(0, n, 16):
        parts = []
        for gi in range(groups):
            blk = q[c0:c0 + 16, gi * group:(gi + 1) * group].reshape(16, quads, 4).transpose(1, 0, 2)
            parts.append(np.ascontiguousarray(blk).reshape(-1).view(np.uint8))
            parts.append(s[c0:c0 + 16, gi].astype(np.float32).view(np.uint8))
            parts.append(o[c0:c0 + 16, gi].astype(np.float32).view(np.uint8))
        panels.append(np.concatenate(parts))
    return panels


def has_vnni512() -> bool:
    try:
        return "avx512_vnni" in Path("/proc/cpuinfo").read_text()
    except OSError:
        return False


def run_quantize16(lib, x16: np.ndarray, group: int):
    k = x16.shape[1]
    groups, quads = k // group, group // 4
    src = np.ascontiguousarray(x16.T)                   # [k][16]
    dst = np.zeros(groups * (quads * 64 + 128), dtype=np.uint8)
    lib.sdasm_quantize16_avx2(ptr(dst), ptr(src), groups, quads, ctypes.c_float(255.0))
    return dst


def run_qgemm(lib, w, x, group: int, y0=None):
    import ref_forms

    m, n = x.shape[0], w.shape[0]
    xq = ref_forms.quantize_inputs(x, group)
    wq = ref_forms.quantize_weights(w, group)
    ap, bp = a_panels(*xq, group), b_panels(*wq, group)
    groups = xq[1].shape[1]
    y = np.zeros((m, n), np.float32) if y0 is None else y0.astype(np.float32).copy()
    for i, a in enumerate(ap):
        for j, b in enumerate(bp):
            c = y[i * 6:, j * 16:]
            lib.sdasm_qgemm_6x16_au_avx512(groups, group // 4, ptr(a), ptr(b),
                                           ctypes.c_void_p(y.ctypes.data + (i * 6 * n + j * 16) * 4), n * 4,
                                           0 if y0 is None else 1)
            del c
    return y


def load_ref():
    import ref_asm

    lib = ctypes.CDLL(str(ref_asm.build()))
    P = ctypes.c_void_p
    lib.refk_mul_mat.argtypes = [P, ctypes.c_int, ctypes.c_int, P, ctypes.c_int, P]
    lib.refk_gated_gelu.argtypes = [P, P, P, ctypes.c_int64]
    lib.refk_exponentials.argtypes = [P, ctypes.c_int64, P, P]
    i64 = ctypes.c_int64
    lib.sdasm_quantize16_avx2.argtypes = [P, P, i64, i64, ctypes.c_float]
    lib.sdasm_qgemm_6x16_au_avx512.argtypes = [i64, i64, P, P, P, i64, i64]
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
    if not has_vnni512():
        print("no AVX512-VNNI here: golden_quant.npz not made")
        return
    qout = {}
    for i, (k, n, m, group) in enumerate(QUANT_CASES):
        w, x = inputs_quant(k, n, m, QUANT_SEED + i)
        qout[f"q16_{i}"] = run_quantize16(lib, x[:16], group)
        qout[f"qmm_{i}"] = run_qgemm(lib, w, x[:m], group)
        if i == 0:
            y0 = np.random.Generator(np.random.PCG64(QUANT_SEED)).uniform(-1, 1, (m, n)).astype(np.float32)
            qout["qmm_acc"] = run_qgemm(lib, w, x[:m], group, y0)
            qout["qmm_acc_y0"] = y0
    qout["cases"] = np.array(QUANT_CASES, dtype=np.int64)
    qout["seed"] = np.array([QUANT_SEED], dtype=np.int64)
    np.savez_compressed(HERE / "golden_quant.npz", **qout)
    print(f"wrote {HERE / 'golden_quant.npz'}")


if __name__ == "__main__":
    main()
