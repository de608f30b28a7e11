"""ctypes binding of ref_forms.c -- TEST INFRASTRUCTURE ONLY (the CPU baseline and a checker).

build() compiles ref_forms.c with gcc (-O3 -march=native -fopenmp) into a
directory of its own, per host CPU (a library built for one CPU may not run on
another's), and loads it.  The functions take and return numpy arrays.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import platform
import subprocess
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "ref_forms.c"

_lib = None


def _cpu_tag() -> str:
    info = platform.processor() or ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags") or line.startswith("model name"):
                    info += line
    except OSError:
        pass
    return hashlib.sha1(info.encode()).hexdigest()[:12]


def build(march: str = "native") -> Path:
    out_dir = Path(os.environ.get("SDB_ORACLE_BUILD", Path(tempfile.gettempdir()) / f"sdb_oracle_{_cpu_tag()}"))
    out_dir.mkdir(parents=True, exist_ok=True)
    lib = out_dir / f"libref_forms_{march.replace('-', '_')}.so"
    if not lib.exists() or lib.stat().st_mtime < SRC.stat().st_mtime:
        cmd = ["gcc", "-O3", f"-march={march}", "-fopenmp", "-shared", "-fPIC", "-o", str(lib), str(SRC), "-lm"]
        subprocess.run(cmd, check=True, capture_output=True)
    return lib


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(str(build()))
        P = ctypes.c_void_p
        i, f = ctypes.c_int, ctypes.c_float
        lib.rf_mul_mat.argtypes = [P, i, i, P, i, P]
        lib.rf_conv2d.argtypes = [P, i, i, i, i, P, i, i, i, i, i, i, i, i, i, P, i, i]
        lib.rf_attention.argtypes = [P, P, P, P, i, i, i, i, i, i, i, f, i, i]
        lib.rf_group_norm.argtypes = [P, P, i, i, ctypes.c_long, i, f, P, P, i]
        lib.rf_qmul_mat.argtypes = [P, i, i, P, i, P, i, i, i, i, i]
        lib.rf_quantize_weights.argtypes = [P, i, i, i, i, i, P, P, P]
        lib.rf_quantize_inputs.argtypes = [P, i, i, i, i, P, P, P]
        lib.rf_qfold.argtypes = [P, P, P, i, P, P, P, i, i, i, P, i]
        lib.rf_threads.restype = i
        lib.rf_set_threads.argtypes = [i]
        _lib = lib
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def threads() -> int:
    return load().rf_threads()


def set_threads(n: int) -> None:
    load().rf_set_threads(n)


def mul_mat(w16: np.ndarray, x: np.ndarray) -> np.ndarray:
    """w16 (N, K) float16, x (M, K) float32 -> (M, N) float32 (mul_mat.cc's form)."""
    w16 = np.ascontiguousarray(w16, dtype=np.float16)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, k = w16.shape
    m = x.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    load().rf_mul_mat(_p(w16), n, k, _p(x), m, _p(y))
    return y


def conv2d(w16, x, stride=(1, 1), padding=(0, 0), dilation=(1, 1), oc_range=None) -> np.ndarray:
    """w16 (OC, IC, KH, KW) float16, x (N, IC, H, W) float32 -> (N, OC, OH, OW) (conv2d.cc's form)."""
    w16 = np.ascontiguousarray(w16, dtype=np.float16)
    x = np.ascontiguousarray(x, dtype=np.float32)
    oc, ic, kh, kw = w16.shape
    n, _, h, wd = x.shape
    oh = (h + 2 * padding[1] - dilation[1] * (kh - 1) - 1) // stride[1] + 1
    ow = (wd + 2 * padding[0] - dilation[0] * (kw - 1) - 1) // stride[0] + 1
    out = np.zeros((n, oc, oh, ow), dtype=np.float32)
    lo, hi = oc_range if oc_range else (0, oc)
    load().rf_conv2d(_p(w16), oc, ic, kh, kw, _p(x), n, h, wd, stride[0], stride[1], padding[0], padding[1],
                     dilation[0], dilation[1], _p(out), lo, hi)
    return out


def attention(q, k, v, heads: int, kv_heads: int, scale: float, q_range=None) -> np.ndarray:
    """q (B, LQ, H*D), k/v (B, LK, HK*D) float32 -> (B, LQ, H*DV) (attention.cc's form)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    b, lq, hd = q.shape
    lk = k.shape[1]
    d = hd // heads
    dv = v.shape[2] // kv_heads
    out = np.zeros((b, lq, heads * dv), dtype=np.float32)
    lo, hi = q_range if q_range else (0, lq)
    load().rf_attention(_p(q), _p(k), _p(v), _p(out), b, lq, lk, heads, kv_heads, d, dv, scale, lo, hi)
    return out


def group_norm(x, groups: int, eps: float, gamma=None, beta=None, silu=False) -> np.ndarray:
    """x (N, C, H, W) float32 -> normalised, with gamma/beta per channel and SiLU (norm.cc's form)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, c = x.shape[:2]
    hw = int(np.prod(x.shape[2:]))
    y = np.empty_like(x)
    g = np.ascontiguousarray(gamma, dtype=np.float32) if gamma is not None else None
    b = np.ascontiguousarray(beta, dtype=np.float32) if beta is not None else None
    load().rf_group_norm(_p(x), _p(y), n, c, hw, groups, eps, _p(g) if g is not None else None,
                         _p(b) if b is not None else None, 1 if silu else 0)
    return y


def qmul_mat(w: np.ndarray, x: np.ndarray, group: int = 64, levels: int = 255, wmax: int = 127,
             weight_groups: bool = True, y0: np.ndarray | None = None) -> np.ndarray:
    """The reference's quantized linear layer (bits = 8, quant.cc's C++ form): w (N, K) float16 or
    float32 (read as float32, which FP16 values are exactly), x (M, K) float32 -> (M, N) float32;
    with y0, the sums start from it (accumulate)."""
    w32 = np.ascontiguousarray(w, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, k = w32.shape
    m = x.shape[0]
    y = np.ascontiguousarray(y0, dtype=np.float32).copy() if y0 is not None else np.empty((m, n), np.float32)
    load().rf_qmul_mat(_p(w32), n, k, _p(x), m, _p(y), group, levels, wmax,
                       1 if weight_groups else 0, 1 if y0 is not None else 0)
    return y


def quantize_inputs(x: np.ndarray, group: int = 64, levels: int = 255):
    """Inputs (M, K) float32 -> (bytes (M, groups * group) uint8, scales (M, groups), offsets (M, groups))."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    groups = -(-k // group)
    q = np.empty((m, groups * group), np.uint8)
    s = np.empty((m, groups), np.float32)
    o = np.empty((m, groups), np.float32)
    load().rf_quantize_inputs(_p(x), m, k, group, levels, _p(q), _p(s), _p(o))
    return q, s, o


def quantize_weights(w: np.ndarray, group: int = 64, wmax: int = 127, weight_groups: bool = True):
    """Weights (N, K) -> (bytes (N, groups * group) int8, scales (N, groups), offsets (N, groups))."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    groups = -(-k // group)
    q = np.empty((n, groups * group), np.int8)
    s = np.empty((n, groups), np.float32)
    o = np.empty((n, groups), np.float32)
    load().rf_quantize_weights(_p(w), n, k, group, wmax, 1 if weight_groups else 0, _p(q), _p(s), _p(o))
    return q, s, o


def qfold(xq, wq, group: int = 64, y0: np.ndarray | None = None) -> np.ndarray:
    """The fold of quantized operands (quantize_inputs' and quantize_weights' triples) -> (M, N) float32."""
    qx, sx, ox = (np.ascontiguousarray(a) for a in xq)
    qw, sw, ow = (np.ascontiguousarray(a) for a in wq)
    m, n, groups = qx.shape[0], qw.shape[0], sx.shape[1]
    y = np.ascontiguousarray(y0, dtype=np.float32).copy() if y0 is not None else np.empty((m, n), np.float32)
    load().rf_qfold(_p(qx), _p(sx), _p(ox), m, _p(qw), _p(sw), _p(ow), n, groups, group, _p(y),
                    1 if y0 is not None else 0)
    return y
