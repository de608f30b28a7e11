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
        lib.rf_expf.argtypes = [P, P, ctypes.c_long]
        lib.rf_norm.argtypes = [P, P, ctypes.c_long, i, ctypes.c_float, P, P]
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


def norm(x, eps: float, gamma=None, beta=None, out=None) -> np.ndarray:
    """Rows (the last dimension) of x float32 normalised, then gamma and beta (norm.cc's form)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x) if out is None else out
    g = np.ascontiguousarray(gamma, dtype=np.float32) if gamma is not None else None
    b = np.ascontiguousarray(beta, dtype=np.float32) if beta is not None else None
    load().rf_norm(_p(x), _p(y), x.size // x.shape[-1], x.shape[-1], eps, _p(g) if g is not None else None,
                   _p(b) if b is not None else None)
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


def _quantize_weights_spans(w, group, wmax, weight_groups, span):
    """quantize_weights with per-row scales over stretches of `span` numbers of k (a multiple of the
    group): each stretch quantized as a row of its own (quant.cc quantize_panel_weights over the
    stretch the caller passes)."""
    k = w.shape[1]
    if weight_groups or span is None or span >= k:
        return quantize_weights(w, group, wmax, weight_groups)
    parts = [quantize_weights(w[:, k0:k0 + span], group, wmax, False) for k0 in range(0, k, span)]
    return tuple(np.concatenate([p[i] for p in parts], axis=1) for i in range(3))


def im2col(x: np.ndarray, kh: int, kw: int, stride=(1, 1), padding=(0, 0), dilation=(1, 1)) -> np.ndarray:
    """The columns of a direct convolution, float32: x (N, IC, H, W) -> (N * OH * OW, IC * KH * KW), the
    positions ow fastest, k = (ic, ky, kx) kx fastest, taps outside the image 0 (conv2d.cc:231-316)."""
    x = np.asarray(x, np.float32)
    n, ic, h, wd = x.shape
    s0, s1 = stride
    p0, p1 = padding
    d0, d1 = dilation
    oh = (h + 2 * p1 - d1 * (kh - 1) - 1) // s1 + 1
    ow = (wd + 2 * p0 - d0 * (kw - 1) - 1) // s0 + 1
    xp = np.zeros((n, ic, h + 2 * p1 + d1 * kh + s1, wd + 2 * p0 + d0 * kw + s0), np.float32)
    xp[:, :, p1:p1 + h, p0:p0 + wd] = x
    cols = np.empty((n, oh, ow, ic, kh, kw), np.float32)
    for ky in range(kh):
        for kx in range(kw):
            patch = xp[:, :, ky * d1:ky * d1 + s1 * (oh - 1) + 1:s1, kx * d0:kx * d0 + s0 * (ow - 1) + 1:s0]
            cols[:, :, :, :, ky, kx] = patch.transpose(0, 2, 3, 1)
    return cols.reshape(n * oh * ow, ic * kh * kw), (n, oh, ow)


def qconv2d(w, x, stride=(1, 1), padding=(0, 0), dilation=(1, 1), group: int = 64, levels: int = 255,
            wmax: int = 127, weight_groups: bool = True) -> np.ndarray:
    """The reference's quantized direct convolution (conv2d.cc:338-470): the kernel as (OC, IC*KH*KW)
    rows, each output position's columns quantized in groups of k, folded as the quantized linear
    layer.  w (OC, IC, KH, KW), x (N, IC, H, W) -> (N, OC, OH, OW) float32, before any chain."""
    oc, ic, kh, kw = w.shape
    cols, (n, oh, ow) = im2col(x, kh, kw, stride, padding, dilation)
    wm = np.asarray(w, np.float32).reshape(oc, ic * kh * kw)
    y = qmul_mat(wm, cols, group, levels, wmax, weight_groups)
    return y.reshape(n, oh, ow, oc).transpose(0, 3, 1, 2).copy()


def winograd2_weights(w) -> np.ndarray:
    """U = G g G^T of every kernel in FP32, the reference's order (winograd.cc:681-729): -> (16, OC, IC)."""
    g = np.asarray(w, np.float32)
    half = np.float32(0.5)
    t = []
    for j in range(3):
        g0, g1, g2 = g[:, :, 0, j], g[:, :, 1, j], g[:, :, 2, j]
        t.append((g0, half * ((g0 + g1) + g2), half * ((g0 - g1) + g2), g2))
    u = []
    for i in range(4):
        a, b, d = t[0][i], t[1][i], t[2][i]
        u += [a, half * ((a + b) + d), half * ((a - b) + d), d]
    return np.stack(u)


def winograd2_inputs(x, padding):
    """B^T d B of every tile in FP32, the reference's order (winograd.cc:440-500, 640-665): the rows of
    the tile by row s of B^T first, then combined by row r; -> ((16, N * TH * TW, IC), (n, th, tw, oh, ow))."""
    x = np.asarray(x, np.float32)
    n, ic, h, wd = x.shape
    p0, p1 = padding
    oh, ow = h + 2 * p1 - 2, wd + 2 * p0 - 2
    th, tw = (oh + 1) // 2, (ow + 1) // 2
    xp = np.zeros((n, ic, 2 * th + 2, 2 * tw + 2), np.float32)
    hh, ww = min(h, 2 * th + 2 - p1), min(wd, 2 * tw + 2 - p0)
    xp[:, :, p1:p1 + hh, p0:p0 + ww] = x[:, :, :hh, :ww]
    d = np.empty((n, ic, th, tw, 4, 4), np.float32)
    for i in range(4):
        for j in range(4):
            d[..., i, j] = xp[:, :, i:i + 2 * th:2, j:j + 2 * tw:2]

    def trow(i, s):
        r = d[..., i, :]
        return [r[..., 0] - r[..., 2], r[..., 1] + r[..., 2], r[..., 2] - r[..., 1], r[..., 1] - r[..., 3]][s]

    v = []
    for r in range(4):
        for s in range(4):
            rows = [trow(i, s) for i in range(4)]
            e = [rows[0] - rows[2], rows[1] + rows[2], rows[2] - rows[1], rows[1] - rows[3]][r]
            v.append(e.transpose(0, 2, 3, 1).reshape(n * th * tw, ic))
    return np.stack(v), (n, th, tw, oh, ow)


def winograd2_outputs(m, shape) -> np.ndarray:
    """Y = A^T M A in FP32, the reference's order (winograd.cc:540-560): m (16, tiles, OC) -> (N, OC, OH, OW)."""
    n, th, tw, oh, ow = shape
    oc = m.shape[2]
    mm = m.reshape(4, 4, n, th, tw, oc)
    a0 = [(mm[0, j] + mm[1, j]) + mm[2, j] for j in range(4)]
    a1 = [(mm[1, j] - mm[2, j]) - mm[3, j] for j in range(4)]
    y = np.empty((n, th, 2, tw, 2, oc), np.float32)
    y[:, :, 0, :, 0] = (a0[0] + a0[1]) + a0[2]
    y[:, :, 0, :, 1] = (a0[1] - a0[2]) - a0[3]
    y[:, :, 1, :, 0] = (a1[0] + a1[1]) + a1[2]
    y[:, :, 1, :, 1] = (a1[1] - a1[2]) - a1[3]
    y = y.reshape(n, 2 * th, 2 * tw, oc)[:, :oh, :ow]
    return y.transpose(0, 3, 1, 2).copy()


def qwinograd2(w, x, padding=(1, 1), group: int = 64, levels: int = 255, wmax: int = 127,
               weight_groups: bool = True, span: int | None = None) -> np.ndarray:
    """The reference's quantized F(2x2, 3x3) (winograd.cc:1826-2100): each xi's transformed kernels
    quantized per output channel in groups of input channels (per-row scales over stretches of `span`
    channels), each tile's transformed inputs likewise, folded, then A^T M A.  -> (N, OC, OH, OW)."""
    u = winograd2_weights(w)
    v, shape = winograd2_inputs(x, padding)
    m = np.stack([qfold(quantize_inputs(v[i], group, levels),
                        _quantize_weights_spans(u[i], group, wmax, weight_groups, span), group) for i in range(16)])
    return winograd2_outputs(m, shape)


def expf(x: np.ndarray) -> np.ndarray:
    """The C library's expf of every element (float32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    load().rf_expf(_p(x), _p(y), x.size)
    return y


def qattention(q, k, v, heads: int, kv_heads: int, scale: float, group: int = 64, levels: int = 255,
               wmax: int = 127) -> np.ndarray:
    """The reference's attention with integer products (attention.cc:596-844).

    q (B, LQ, H*D), k (B, LK, HK*D), v (B, LK, HK*DV) -> (B, LQ, H*DV) float32.  Per head: the queries
    quantized (unsigned, zero point) and the keys (signed), each over its D numbers as one group of
    4 ceil(D/4), the queries' scales and offsets times the softmax's scale (FP32); the scores their fold;
    each query's exponentials of its scores less their greatest -- the reference's exponential for the
    keys before the last LK % 8, the C library's expf for those -- summed in double; the exponentials
    quantized per group of keys, the values per dimension per group of keys; their fold times
    float(1 / sum).  Head h reads key head h / (H / HK).
    """
    import oracle

    f32 = np.float32
    b, lq, hd = q.shape
    lk = k.shape[1]
    d = hd // heads
    dv = v.shape[2] // kv_heads
    gd = 4 * (-(-d // 4))
    tail0 = lk - lk % 8
    out = np.empty((b, lq, heads * dv), f32)
    for bi in range(b):
        for h in range(heads):
            hk = h // (heads // kv_heads)
            qm = np.ascontiguousarray(q[bi, :, h * d:(h + 1) * d], dtype=f32)
            km = np.ascontiguousarray(k[bi, :, hk * d:(hk + 1) * d], dtype=f32)
            vm = np.ascontiguousarray(v[bi, :, hk * dv:(hk + 1) * dv], dtype=f32)
            qx, sx, ox = quantize_inputs(qm, gd, levels)
            sx, ox = (sx * f32(scale)).astype(f32), (ox * f32(scale)).astype(f32)
            s = qfold((qx, sx, ox), quantize_weights(km, gd, wmax, True), gd)
            x = (s - s.max(axis=1, keepdims=True)).astype(f32)
            e = np.empty_like(x)
            e[:, :tail0] = oracle.exponential(x[:, :tail0])
            e[:, tail0:] = expf(x[:, tail0:])
            rec = (1.0 / e.astype(np.float64).sum(axis=1)).astype(f32)
            o = qfold(quantize_inputs(e, group, levels), quantize_weights(vm.T, group, wmax, True), group)
            out[bi, :, h * dv:(h + 1) * dv] = (o * rec[:, None]).astype(f32)
    return out
