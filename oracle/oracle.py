"""CPU oracle of the reference's operations -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this module, and only as the checker (or the timed CPU baseline),
never as the thing measured or shipped.

It restates, in float64 numpy, what the reference's own test harness
(tests/ops_test.cc) computes as the exact result of each operation from the
same FP16/FP32 inputs, and the measure it judges every form by:

    error(i) = |out[i] - exact[i]| / sum over the products of |product|

(ops_test.cc:9-25, 186-200; the magnitude of an output is the sum of the
magnitudes of the products summed into it).  The reference's bounds:
kSingle = 1e-5 for single-precision forms (ops_test.cc:157), kQuantized =
1e-2 for the 8-bit forms (ops_test.cc:223), fused vs apart within 1e-6 of the
largest output (ops_test.cc:568-597).

Each function cites the lines of the reference it restates.  Layouts are the
torch ones of the binding: a ggml tensor ne = [d0, d1, d2, d3] is the numpy
array of shape (d3, d2, d1, d0).
"""
from __future__ import annotations

import math

import numpy as np

K_SINGLE = 1e-5          # ops_test.cc:157
K_QUANTIZED = 1e-2       # ops_test.cc:223
K_FUSED_APART = 1e-6     # ops_test.cc:568-597
SEED = 20261011          # ops_test.cc:61-64

# The bound this build holds its FP32-activation paths to (the north star's).
K_B200 = 1e-6


def metric(out: np.ndarray, exact: np.ndarray, magnitude: np.ndarray) -> float:
    """The worst error relative to the magnitudes summed (ops_test.cc:186-200).

    A magnitude of 0 counts as 1; a non-finite error is infinite, which is how
    the NaN canary of unwritten outputs fails (ops_test.cc:108-110).
    """
    out = np.asarray(out, dtype=np.float64).reshape(-1)
    exact = np.asarray(exact, dtype=np.float64).reshape(-1)
    mag = np.asarray(magnitude, dtype=np.float64).reshape(-1)
    scale = np.where(mag > 0, mag, 1.0)
    e = np.abs(out - exact) / scale
    if not np.all(np.isfinite(e)):
        return math.inf
    return float(e.max()) if e.size else 0.0


def as64(a) -> np.ndarray:
    return np.asarray(a).astype(np.float64)


# ---------------------------------------------------------------- mul_mat

def mul_mat_exact(w, x):
    """Exact dst[..., n] = sum_k w[n, k] x[..., k] and its magnitude (ops_test.cc:450-461).

    w (N, K) FP16/FP32, x (..., K) FP32.  Each product of an FP32 and an
    FP16/FP32 number is exact in double; the sums are double.
    """
    w64, x64 = as64(w), as64(x)
    exact = x64 @ w64.T
    magnitude = np.abs(x64) @ np.abs(w64).T
    return exact, magnitude


def mul_mat_f32_running(w, x):
    """The reference's single-precision form of a product: each output a running
    FP32 sum over k of FP32 products (the micro-kernel's FMA chain over k-stretches,
    mul_mat.cc:306-366, microkernel.cc:51-69).  x (M, K), w (N, K) -> (M, N)."""
    x32 = np.asarray(x, dtype=np.float32)
    w32 = np.asarray(w, dtype=np.float32)
    acc = np.zeros((x32.shape[0], w32.shape[0]), dtype=np.float32)
    for k in range(x32.shape[1]):
        # An FMA rounds once: the product of a float and an FP16 value is exact in double.
        acc = (acc.astype(np.float64) + np.outer(x32[:, k], w32[:, k])).astype(np.float32)
    return acc


def gated_exact(w, x, bias):
    """Exact GEGLU after a linear layer and its magnitude (ops_test.cc:722-768).

    y = x w^T + b split into halves x | gate along the last dimension; out =
    y_x * GELU(y_gate), GELU by tanh in double; magnitude = |sum_x| GELU(g)
    + |y_x| * 1.13 * |sum_g| (d/dv GELU within [-0.13, 1.13]).
    """
    w64, x64, b64 = as64(w), as64(x), as64(bias)
    half = w64.shape[0] // 2
    s = x64 @ w64.T + b64
    m = np.abs(x64) @ np.abs(w64).T + np.abs(b64)
    sx, sg = s[..., :half], s[..., half:]
    mx, mg = m[..., :half], m[..., half:]
    g = 0.5 * sg * (1.0 + np.tanh(0.79788456080286535587989211986876 * (sg + 0.044715 * sg ** 3)))
    return sx * g, mx * np.abs(g) + np.abs(sx) * 1.13 * mg


# ---------------------------------------------------------------- conv2d

def conv_out(size, k, s, p, d):
    return (size + 2 * p - d * (k - 1) - 1) // s + 1


def conv2d_exact(w, x, stride=(1, 1), padding=(0, 0), dilation=(1, 1)):
    """Exact direct convolution and its magnitude (ops_test.cc:385-424).

    w (OC, IC, KH, KW), x (N, IC, H, W) -> (N, OC, OH, OW); stride, padding
    and dilation are (dim 0 = width, dim 1 = height) as ggml's s0/s1 etc.
    Out-of-image taps contribute nothing.
    """
    w64, x64 = as64(w), as64(x)
    oc, ic, kh, kw = w64.shape
    n, _, h, wd = x64.shape
    s0, s1 = stride
    p0, p1 = padding
    d0, d1 = dilation
    oh, ow = conv_out(h, kh, s1, p1, d1), conv_out(wd, kw, s0, p0, d0)
    xp = np.zeros((n, ic, h + 2 * p1 + d1 * kh + s1, wd + 2 * p0 + d0 * kw + s0))
    xp[:, :, p1:p1 + h, p0:p0 + wd] = x64
    cols = np.empty((n, oh, ow, ic, kh, kw))
    for ky in range(kh):
        for kx in range(kw):
            ys = ky * d1
            xs = kx * d0
            patch = xp[:, :, ys:ys + s1 * (oh - 1) + 1:s1, xs:xs + s0 * (ow - 1) + 1:s0]  # (n, ic, oh, ow)
            cols[:, :, :, :, ky, kx] = patch.transpose(0, 2, 3, 1)
    cols = cols.reshape(n * oh * ow, ic * kh * kw)
    wm = w64.reshape(oc, ic * kh * kw)
    exact = (cols @ wm.T).reshape(n, oh, ow, oc).transpose(0, 3, 1, 2)
    magnitude = (np.abs(cols) @ np.abs(wm).T).reshape(n, oh, ow, oc).transpose(0, 3, 1, 2)
    return exact, magnitude


# ---------------------------------------------------------------- Winograd

# F(2x2, 3x3): winograd.cc:14-22.  F(4x4, 3x3), points 0, 1, -1, 2, -1/2, inf:
# winograd.cc:1155-1190 (B^T, A^T) and 1259-1264 (G, as the reference's float
# constants).
WINO_BT2 = np.array([[1, 0, -1, 0], [0, 1, 1, 0], [0, -1, 1, 0], [0, 1, 0, -1]], np.float32)
WINO_G2 = np.array([[1, 0, 0], [0.5, 0.5, 0.5], [0.5, -0.5, 0.5], [0, 0, 1]], np.float32)
WINO_AT2 = np.array([[1, 1, 1, 0], [0, 1, -1, -1]], np.float32)
WINO_BT4 = np.array([[1, 1.5, -2, -1.5, 1, 0], [0, -1, -2.5, -0.5, 1, 0], [0, 1, 0.5, -2.5, 1, 0],
                     [0, -0.5, -1, 0.5, 1, 0], [0, 2, -1, -2, 1, 0], [0, 1, 1.5, -2, -1.5, 1]], np.float32)
WINO_G4 = np.array([[1, 0, 0], [np.float32(-1.0) / np.float32(3)] * 3,
                    [np.float32(1.0) / np.float32(3), np.float32(-1.0) / np.float32(3), np.float32(1.0) / np.float32(3)],
                    [np.float32(1.0) / np.float32(15), np.float32(2.0) / np.float32(15), np.float32(4.0) / np.float32(15)],
                    [np.float32(-16.0) / np.float32(15), np.float32(8.0) / np.float32(15), np.float32(-4.0) / np.float32(15)],
                    [0, 0, 1]], np.float32)
WINO_AT4 = np.array([[1, 1, 1, 1, 1, 0], [0, 1, -1, 2, -0.5, 0], [0, 1, 1, 4, 0.25, 0],
                     [0, 1, -1, 8, -0.125, 1]], np.float32)


def winograd_f32(w, x, padding=(1, 1), f: int = 4):
    """The reference's single-precision Winograd form of a 3x3, stride-1 convolution.

    Y = A^T [sum over ic of (G g G^T) (.) (B^T d B)] A per tile of f x f outputs
    (winograd.cc:9-31, 1148-1190), every transform and the channel sums in
    float32 as the reference computes them (transform_weights4 winograd.cc:1266-1300:
    G g then (G g) G^T; the inputs' B^T d B and the outputs' A^T M A likewise).
    The summation order of the channel sums is numpy's, not the micro-kernel's;
    the result's error against conv2d_exact is the size of the reference's own
    (F(4x4): about 7e-7 of the magnitudes at worst, winograd.cc:1165-1168).
    w (OC, IC, 3, 3), x (N, IC, H, W) -> (N, OC, OH, OW).
    """
    bt, g, at = (WINO_BT2, WINO_G2, WINO_AT2) if f == 2 else (WINO_BT4, WINO_G4, WINO_AT4)
    a = bt.shape[0]
    x32 = np.asarray(x, dtype=np.float32)
    w32 = np.asarray(w, dtype=np.float32)
    n, ic, h, wd = x32.shape
    oc = w32.shape[0]
    p0, p1 = padding
    oh, ow = h + 2 * p1 - 2, wd + 2 * p0 - 2
    th, tw = -(-oh // f), -(-ow // f)
    xp = np.zeros((n, ic, th * f + 2, tw * f + 2), np.float32)
    hh, ww = min(h, th * f + 2 - p1), min(wd, tw * f + 2 - p0)
    xp[:, :, p1:p1 + hh, p0:p0 + ww] = x32[:, :, :hh, :ww]
    d = np.stack([np.stack([xp[:, :, i * f:i * f + a, j * f:j * f + a] for j in range(tw)], 1)
                  for i in range(th)], 1)                      # (n, th, tw, ic, a, a)
    v = np.einsum("ij,ntwcjk->ntwcik", bt, d, dtype=np.float32)
    v = np.einsum("ntwcik,lk->ntwcil", v, bt, dtype=np.float32)
    u = np.einsum("ij,ocjk->ocik", g, w32, dtype=np.float32)
    u = np.einsum("ocik,lk->ocil", u, g, dtype=np.float32)
    m = np.einsum("ntwcij,ocij->ntwoij", v, u, dtype=np.float32)
    y = np.einsum("ij,ntwojk->ntwoik", at, m, dtype=np.float32)
    y = np.einsum("ntwoik,lk->ntwoil", y, at, dtype=np.float32)
    return y.transpose(0, 3, 1, 4, 2, 5).reshape(n, oc, th * f, tw * f)[:, :, :oh, :ow]


# ---------------------------------------------------------------- attention

def attention_exact(q, k, v, heads: int, kv_heads: int, scale: float):
    """Exact attention and its magnitude (ops_test.cc:497-534).

    q (B, LQ, H*D), k (B, LK, HK*D), v (B, LK, HK*DV) -> (B, LQ, H*DV).  Scores
    in double scaled by `scale` (an FP32 number), softmax with exp in double,
    each output the sum of w/total * v; its magnitude the sum of |w/total * v|.
    Heads share keys in groups of H/HK (head h uses key head h / (H/HK)).
    """
    q64, k64, v64 = as64(q), as64(k), as64(v)
    b, lq, hd = q64.shape
    lk = k64.shape[1]
    d = hd // heads
    dv = v64.shape[2] // kv_heads
    group = heads // kv_heads
    out = np.empty((b, lq, heads * dv))
    mag = np.empty_like(out)
    sc = float(np.float32(scale))
    for bi in range(b):
        for h in range(heads):
            hk = h // group
            qh = q64[bi, :, h * d:(h + 1) * d]
            kh = k64[bi, :, hk * d:(hk + 1) * d]
            vh = v64[bi, :, hk * dv:(hk + 1) * dv]
            s = (qh @ kh.T) * sc
            s = np.exp(s - s.max(axis=1, keepdims=True))
            p = s / s.sum(axis=1, keepdims=True)
            out[bi, :, h * dv:(h + 1) * dv] = p @ vh
            mag[bi, :, h * dv:(h + 1) * dv] = p @ np.abs(vh)
    return out, mag


# ---------------------------------------------------------------- norms

def _sum_double_lanes(x32: np.ndarray) -> float:
    """row_sum of norm.cc:42-59: 8 double partial sums, the tail, then the partials."""
    n = x32.size
    whole = n // 8 * 8
    parts = np.zeros(8)
    if whole:
        parts = x32[:whole].astype(np.float64).reshape(-1, 8).sum(axis=0)  # order within a lane is immaterial at 1e-16
    s = float(x32[whole:].astype(np.float64).sum())
    for p in parts:
        s += p
    return s


def group_norm_ref(x, groups: int, eps: float):
    """The reference's group normalisation (norm.cc:100-140), in its precision.

    x (N, C, H, W) FP32.  Per (image, group of ceil(C/groups) channels): mean =
    float(sum in double / count); variance = float(sum of float squares of
    float (x - mean) in double / count); y = (x - mean) * float(1 / sqrt(var + eps)).
    """
    x32 = np.asarray(x, dtype=np.float32)
    n, c = x32.shape[:2]
    per = (c + groups - 1) // groups
    y = np.empty_like(x32)
    for i in range(n):
        for g in range(groups):
            c0, c1 = g * per, min(c, (g + 1) * per)
            if c0 >= c1:
                continue
            grp = x32[i, c0:c1].reshape(-1)
            count = grp.size
            mean = np.float32(_sum_double_lanes(grp) / count)
            dev = (grp - mean).astype(np.float32)
            var = np.float32(_sum_double_lanes((dev * dev).astype(np.float32)) / count)
            scale = np.float32(1.0) / np.sqrt(np.float32(var + np.float32(eps)), dtype=np.float32)
            y[i, c0:c1] = ((x32[i, c0:c1] - mean) * scale).astype(np.float32)
    return y


def norm_ref(x, eps: float):
    """The reference's layer normalisation of rows (norm.cc:148-175), in its precision."""
    x32 = np.asarray(x, dtype=np.float32)
    rows = x32.reshape(-1, x32.shape[-1])
    y = np.empty_like(rows)
    for r in range(rows.shape[0]):
        row = rows[r]
        mean = np.float32(_sum_double_lanes(row) / row.size)
        dev = (row - mean).astype(np.float32)
        var = np.float32(_sum_double_lanes((dev * dev).astype(np.float32)) / row.size)
        scale = np.float32(1.0) / np.sqrt(np.float32(var + np.float32(eps)), dtype=np.float32)
        y[r] = ((row - mean) * scale).astype(np.float32)
    return y.reshape(x32.shape)


def group_norm_exact(x, groups: int, eps: float):
    """Group normalisation in double (for the north star's PSNR-style checks)."""
    x64 = as64(x)
    n, c = x64.shape[:2]
    per = (c + groups - 1) // groups
    y = np.empty_like(x64)
    for g in range(groups):
        c0, c1 = g * per, min(c, (g + 1) * per)
        if c0 >= c1:
            continue
        grp = x64[:, c0:c1].reshape(n, -1)
        mean = grp.mean(axis=1)
        var = ((grp - mean[:, None]) ** 2).mean(axis=1)
        y[:, c0:c1] = ((x64[:, c0:c1].reshape(n, -1) - mean[:, None]) / np.sqrt(var[:, None] + eps)).reshape(
            x64[:, c0:c1].shape)
    return y


# ---------------------------------------------------------------- scalar math

def exponential(x):
    """scalar_math.h:34-51 in float32: clamp, n = round(x / ln 2), two-part reduction, Cephes polynomial, 2^n."""
    x = np.minimum(np.maximum(np.asarray(x, dtype=np.float32), np.float32(-87.3)), np.float32(88.73))
    magic = np.float32(12582912.0)
    f = np.float32
    z = (x.astype(np.float64) * float(f(1.44269504088896341)) + 12582912.0).astype(np.float32)  # fmaf: exact product, one rounding
    n = (z - magic).astype(np.float32)
    r = (n.astype(np.float64) * -0.693359375 + x).astype(np.float32)
    r = (n.astype(np.float64) * float(f(2.12194440e-4)) + r).astype(np.float32)
    p = np.full_like(r, f(1.9875691500e-4))
    for c in (1.3981999507e-3, 8.3334519073e-3, 4.1665795894e-2, 1.6666665459e-1, 5.0000001201e-1):
        p = (p.astype(np.float64) * r + float(f(c))).astype(np.float32)
    pr = (p * r).astype(np.float32)
    p = ((pr.astype(np.float64) * r + r).astype(np.float32) + f(1.0)).astype(np.float32)
    e = ((z.view(np.int32) - np.int32(0x4b400000) + np.int32(127)).astype(np.uint32) << np.uint32(23)).view(np.float32)
    return (p * e).astype(np.float32)


def silu(x):
    """scalar_math.h:54-56."""
    x = np.asarray(x, dtype=np.float32)
    return (x / (np.float32(1.0) + exponential(-x))).astype(np.float32)


def gelu(x):
    """scalar_math.h:60-63."""
    x = np.asarray(x, dtype=np.float32)
    y = (x * ((np.float32(0.044715) * x).astype(np.float64) * x + 1.0).astype(np.float32)).astype(np.float32)
    return (x / (np.float32(1.0) + exponential(np.float32(-1.5957691216057308) * y))).astype(np.float32)


def apply_chain(y, steps):
    """Epilogue::apply (fusion.cc:77-86): steps [(kind, operand broadcastable to y)] in order, FP32."""
    y = np.asarray(y, dtype=np.float32).copy()
    for kind, operand in steps:
        if kind == "silu":
            y = silu(y)
        elif kind == "add":
            y = (y + np.asarray(operand, dtype=np.float32)).astype(np.float32)
        elif kind == "mul":
            y = (y * np.asarray(operand, dtype=np.float32)).astype(np.float32)
        else:
            raise ValueError(kind)
    return y


# ---------------------------------------------------------------- fixtures

def generator(seed: int = SEED) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def uniform(rng: np.random.Generator, shape, scale: float, dtype=np.float32) -> np.ndarray:
    """U(-scale, scale) rounded to dtype: the reference's fills (ops_test.cc:66-79)."""
    return rng.uniform(-scale, scale, size=shape).astype(np.float32).astype(dtype)
