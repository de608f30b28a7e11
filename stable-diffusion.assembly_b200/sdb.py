"""Python host binding of libsdb.so: the reference's op interface over the C ABI.

The reference (stable-diffusion.assembly) exposes its kernels to ggml as
operations on ggml tensors (sources/ops.h:26-62): mul_mat, the gated GELU
after it, conv2d (direct or Winograd), attention, group_norm and norm, each
with the chain of element-wise nodes fused after it (sources/fusion.h).
This module offers the same operations on CUDA tensors (torch is used only to
hold device memory and name a stream), described to the library in ggml's
terms: ne[] dimension 0 fastest, nb[] byte strides.  A torch tensor of shape
(d3, d2, d1, d0) is the ggml tensor ne = [d0, d1, d2, d3].

Errors are raised as SdbError with the library's status and message; a
status of NOT_SUPPORTED means the reference would leave the node to ggml.
There is no CPU fallback: without the built library every call raises.
"""
from __future__ import annotations

import ctypes
import os
import weakref
from pathlib import Path
from typing import Iterable, Sequence

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libsdb.so"

TYPE_F32 = 0
TYPE_F16 = 1
STEP_ADD, STEP_MUL, STEP_SILU = 0, 1, 2
MAX_STEPS = 6

OK, NOT_SUPPORTED, INVALID, CUDA_ERROR, OUT_OF_MEMORY, DEVICE_ERROR = range(6)
STATUS_NAMES = ["OK", "NOT_SUPPORTED", "INVALID", "CUDA_ERROR", "OUT_OF_MEMORY", "DEVICE_ERROR"]

# Exported symbols of include/sdb.h, checked by the tests.
EXPORTS = [
    "sdb_mul_mat_supported", "sdb_mul_mat", "sdb_mul_mat_transient", "sdb_mul_mat_gated_supported",
    "sdb_mul_mat_gated",
    "sdb_conv2d_supported", "sdb_conv2d", "sdb_attention_supported", "sdb_attention",
    "sdb_group_norm", "sdb_group_norm_no_alloc", "sdb_norm", "sdb_forget", "sdb_store_stats", "sdb_token_downsampling",
    "sdb_set_tuning", "sdb_get_tuning", "sdb_device_status", "sdb_last_error", "sdb_launch_count",
    "sdb_concat", "sdb_upscale_nearest", "sdb_timestep_embedding", "sdb_euler_cfg_step", "sdb_soft_max",
    "sdb_coarser_tokens", "sdb_euler_ancestral_cfg_step", "sdb_group_norm_stats", "sdb_conv2d_normed",
    "sdb_mul_mat_normed", "sdb_mul_mat_layer_normed", "sdb_mul_mat_gated_layer_normed",
]


class SdbError(RuntimeError):
    def __init__(self, status: int, message: str):
        self.status = status
        name = STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else str(status)
        super().__init__(f"{name}: {message}")


class Tensor(ctypes.Structure):
    _fields_ = [("type", ctypes.c_int32), ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_int64 * 4),
                ("data", ctypes.c_void_p)]


class Step(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("operand", ctypes.c_void_p), ("nb", ctypes.c_int64 * 4)]


class NormIn(ctypes.Structure):
    _fields_ = [("stats", ctypes.c_void_p), ("gamma", ctypes.c_void_p), ("beta", ctypes.c_void_p),
                ("groups", ctypes.c_int32), ("silu", ctypes.c_int32)]


class ChainStruct(ctypes.Structure):
    _fields_ = [("count", ctypes.c_int32), ("steps", Step * MAX_STEPS), ("redirect", ctypes.c_void_p),
                ("from_redirect", ctypes.c_int32)]


_lib = None


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Loads libsdb.so (built by build.py); raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise SdbError(CUDA_ERROR, f"{p} is not built (run stable-diffusion.assembly_b200/build.py)")
    lib = ctypes.CDLL(str(p))
    T = ctypes.POINTER(Tensor)
    C = ctypes.POINTER(ChainStruct)
    vp = ctypes.c_void_p
    i = ctypes.c_int
    sigs = {
        "sdb_mul_mat_supported": (i, [T, T, T]),
        "sdb_mul_mat": (i, [T, T, T, C, vp]),
        "sdb_mul_mat_transient": (i, [T, T, T, C, vp]),
        "sdb_soft_max": (i, [T, T, ctypes.c_float, vp]),
        "sdb_mul_mat_gated_supported": (i, [T, T, T]),
        "sdb_mul_mat_gated": (i, [T, T, T, C, vp]),
        "sdb_conv2d_supported": (i, [T, T, T, ctypes.POINTER(ctypes.c_int32)]),
        "sdb_conv2d": (i, [T, T, T, ctypes.POINTER(ctypes.c_int32), C, vp]),
        "sdb_attention_supported": (i, [T, T, T, T]),
        "sdb_attention": (i, [T, T, T, T, ctypes.c_float, C, vp]),
        "sdb_group_norm": (i, [T, T, ctypes.c_int32, ctypes.c_float, C, vp]),
        "sdb_group_norm_no_alloc": (i, [T, T, ctypes.c_int32, ctypes.c_float, C, vp]),
        "sdb_norm": (i, [T, T, ctypes.c_float, C, vp]),
        "sdb_forget": (None, [vp, ctypes.c_size_t]),
        "sdb_store_stats": (None, [ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]),
        "sdb_token_downsampling": (i, [ctypes.c_int64, ctypes.c_int64]),
        "sdb_set_tuning": (i, [ctypes.c_char_p]),
        "sdb_get_tuning": (i, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)]),
        "sdb_device_status": (ctypes.c_uint, [i]),
        "sdb_last_error": (ctypes.c_char_p, []),
        "sdb_launch_count": (ctypes.c_uint64, []),
        "sdb_concat": (i, [T, T, T, ctypes.c_int32, vp]),
        "sdb_upscale_nearest": (i, [T, T, vp]),
        "sdb_coarser_tokens": (i, [T, T, ctypes.c_int32, vp]),
        "sdb_timestep_embedding": (i, [T, T, ctypes.c_int32, ctypes.c_int32, vp]),
        "sdb_group_norm_stats": (i, [T, ctypes.c_int32, ctypes.c_float, vp, vp]),
        "sdb_conv2d_normed": (i, [T, T, T, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(NormIn), C, vp]),
        "sdb_mul_mat_normed": (i, [T, T, T, ctypes.POINTER(NormIn), C, vp]),
        "sdb_mul_mat_layer_normed": (i, [T, T, T, ctypes.c_float, C, C, vp]),
        "sdb_mul_mat_gated_layer_normed": (i, [T, T, T, ctypes.c_float, C, C, vp]),
        "sdb_euler_cfg_step": (i, [vp, vp, vp, ctypes.c_int64, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                   ctypes.c_float, vp]),
        "sdb_euler_ancestral_cfg_step": (i, [vp, vp, vp, vp, ctypes.c_int64, ctypes.c_float, ctypes.c_float,
                                             ctypes.c_float, ctypes.c_float, vp]),
    }
    for name, (res, args) in sigs.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    _lib = lib
    return lib


def _check(status: int) -> None:
    if status != OK:
        msg = load().sdb_last_error()
        raise SdbError(status, msg.decode() if msg else "")


# ---------------------------------------------------------------- tensors

def describe(t, ne: Sequence[int] | None = None, nb: Sequence[int] | None = None) -> Tensor:
    """The ggml description of a torch tensor (or an explicit ne / nb view of it)."""
    import torch

    if t.dtype == torch.float32:
        ty, es = TYPE_F32, 4
    elif t.dtype == torch.float16:
        ty, es = TYPE_F16, 2
    else:
        raise SdbError(INVALID, f"unsupported dtype {t.dtype}")
    d = Tensor()
    d.type = ty
    if ne is None:
        shape = list(reversed(t.shape))
        strides = [s * es for s in reversed(t.stride())]
        while len(shape) < 4:
            strides.append(strides[-1] * shape[-1] if shape else es)
            shape.append(1)
        if len(shape) > 4:
            raise SdbError(INVALID, "more than 4 dimensions")
        ne, nb = shape, strides
    for k in range(4):
        d.ne[k] = int(ne[k])
        d.nb[k] = int(nb[k])
    d.data = t.data_ptr()
    return d


def _stream_ptr(stream) -> int:
    import torch

    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream)


class Chain:
    """An epilogue chain (sdasm::Epilogue): steps applied in order to each output element.

    add(t) / mul(t): t an FP32 CUDA tensor broadcastable to the output in ggml's
    sense (a dimension of extent 1 is broadcast); silu().  redirect(r,
    from_redirect) makes the operation write into r (a residual connection).
    """

    def __init__(self):
        self.steps: list[tuple[int, object, list[int]]] = []
        self.redirect_tensor = None
        self.from_redirect = False
        self._keep: list = []

    def _operand(self, kind, t, nb):
        import torch

        if t.dtype != torch.float32 or not t.is_cuda:
            raise SdbError(INVALID, "chain operands are FP32 CUDA tensors")
        if nb is None:
            shape = list(reversed(t.shape)) + [1] * (4 - t.dim())
            strides = list(reversed(t.stride())) + [0] * (4 - t.dim())
            nb = [0 if shape[k] == 1 else strides[k] for k in range(4)]
        self.steps.append((kind, t, list(nb)))
        return self

    def add(self, t, nb=None):
        return self._operand(STEP_ADD, t, nb)

    def mul(self, t, nb=None):
        return self._operand(STEP_MUL, t, nb)

    def silu(self):
        self.steps.append((STEP_SILU, None, [0, 0, 0, 0]))
        return self

    def redirect(self, t, from_redirect: bool = False):
        self.redirect_tensor = t
        self.from_redirect = from_redirect
        return self

    def struct(self) -> ChainStruct:
        if len(self.steps) > MAX_STEPS:
            raise SdbError(INVALID, "chain longer than 6 steps")
        c = ChainStruct()
        c.count = len(self.steps)
        for i, (kind, t, nb) in enumerate(self.steps):
            c.steps[i].kind = kind
            c.steps[i].operand = t.data_ptr() if t is not None else None
            for k in range(4):
                c.steps[i].nb[k] = nb[k]
        c.redirect = self.redirect_tensor.data_ptr() if self.redirect_tensor is not None else None
        c.from_redirect = 1 if self.from_redirect else 0
        return c


def _chain_ptr(chain: Chain | None):
    if chain is None:
        return None
    return ctypes.pointer(chain.struct())


# ---------------------------------------------------------------- weights

# The library keeps weights packed by address (the reference's store, which
# ggml tells of every write through sdasm_forget).  torch's caching allocator
# hands a freed block's address to the next tensor, so the binding forgets an
# address when a different tensor object shows up there.  A weight changed in
# place must still be forgotten by the caller: forget(w).
_weights: dict[int, weakref.ref] = {}


def _guard_weight(w) -> None:
    ptr = w.data_ptr()
    ref = _weights.get(ptr)
    if ref is not None and ref() is w:
        return
    if ref is not None:
        load().sdb_forget(ctypes.c_void_p(ptr), ctypes.c_size_t(w.numel() * w.element_size()))
    _weights[ptr] = weakref.ref(w)


# ---------------------------------------------------------------- operations

def mul_mat(w, x, out=None, chain: Chain | None = None, stream=None):
    """dst[m][n] = sum_k x[m][k] w[n][k]: w (N, K) FP16/FP32, x (..., K) FP32 -> (..., N)."""
    import torch

    lib = load()
    if out is None:
        out = torch.empty(*x.shape[:-1], w.shape[0], dtype=torch.float32, device=x.device)
    _guard_weight(w)
    dw, dx, dy = describe(w), describe(x), describe(out)
    if not lib.sdb_mul_mat_supported(dw, dx, dy):
        raise SdbError(NOT_SUPPORTED, "mul_mat shapes not supported")
    _check(lib.sdb_mul_mat(dw, dx, dy, _chain_ptr(chain), ctypes.c_void_p(_stream_ptr(stream))))
    return out


def mul_mat_transient(w, x, out=None, chain: Chain | None = None, stream=None):
    """mul_mat for a first operand written between calls (packed every call, never kept):
    w (N, K) FP32/FP16, x (..., K) FP32 -> (..., N)."""
    import torch

    lib = load()
    if out is None:
        out = torch.empty(*x.shape[:-1], w.shape[0], dtype=torch.float32, device=x.device)
    _check(lib.sdb_mul_mat_transient(describe(w), describe(x), describe(out), _chain_ptr(chain),
                                     ctypes.c_void_p(_stream_ptr(stream))))
    return out


def soft_max(x, scale: float = 1.0, out=None, stream=None):
    """GGML_OP_SOFT_MAX without a mask: softmax(scale * x) along the last dimension (x may be out)."""
    import torch

    lib = load()
    if out is None:
        out = torch.empty_like(x)
    _check(lib.sdb_soft_max(describe(x), describe(out), ctypes.c_float(scale), ctypes.c_void_p(_stream_ptr(stream))))
    return out


def mul_mat_supported(w, x, out) -> bool:
    """Whether sdb_mul_mat takes these operands (under the tuning in effect)."""
    return bool(load().sdb_mul_mat_supported(describe(w), describe(x), describe(out)))


def mul_mat_gated_supported(w, x, out) -> bool:
    """Whether sdb_mul_mat_gated takes these operands (under the tuning in effect)."""
    return bool(load().sdb_mul_mat_gated_supported(describe(w), describe(x), describe(out)))


def mul_mat_gated(w, x, out=None, chain: Chain | None = None, stream=None):
    """GEGLU: y = x w^T (+chain), out = y[..., :N/2] * GELU(y[..., N/2:])."""
    import torch

    lib = load()
    if out is None:
        out = torch.empty(*x.shape[:-1], w.shape[0] // 2, dtype=torch.float32, device=x.device)
    _guard_weight(w)
    dw, dx, dy = describe(w), describe(x), describe(out)
    _check(lib.sdb_mul_mat_gated(dw, dx, dy, _chain_ptr(chain), ctypes.c_void_p(_stream_ptr(stream))))
    return out


def conv_out_size(size: int, k: int, s: int, p: int, d: int) -> int:
    return (size + 2 * p - d * (k - 1) - 1) // s + 1


def conv2d(w, x, stride=(1, 1), padding=(0, 0), dilation=(1, 1), out=None, chain: Chain | None = None,
           stream=None):
    """ggml_conv_2d_direct: w (OC, IC, KH, KW), x (N, IC, H, W) FP32 -> (N, OC, OH, OW)."""
    import torch

    lib = load()
    oc, _, kh, kw = w.shape
    n, _, h, wd = x.shape
    oh = conv_out_size(h, kh, stride[1], padding[1], dilation[1])
    ow = conv_out_size(wd, kw, stride[0], padding[0], dilation[0])
    if out is None:
        out = torch.empty(n, oc, oh, ow, dtype=torch.float32, device=x.device)
    params = (ctypes.c_int32 * 6)(stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1])
    _guard_weight(w)
    dw, dx, dy = describe(w), describe(x), describe(out)
    _check(lib.sdb_conv2d(dw, dx, dy, params, _chain_ptr(chain), ctypes.c_void_p(_stream_ptr(stream))))
    return out


def attention(q, k, v, scale: float, out=None, chain: Chain | None = None, stream=None):
    """FLASH_ATTN_EXT without a mask on token-major tensors.

    q (B, LQ, H*D), k (B, LK, HK*D), v (B, LK, HK*DV) with D / DV given by the
    head counts in `heads` of the views below; returns (B, LQ, H*DV).
    Use attention_heads() for explicit head counts.
    """
    raise NotImplementedError("use attention_heads(q, k, v, heads, kv_heads, scale)")


def attention_heads(q, k, v, heads: int, kv_heads: int, scale: float, out=None, chain: Chain | None = None,
                    stream=None):
    """softmax(scale q k^T) v per head; q (B, LQ, H*D), k/v (B, LK, HK*D) -> (B, LQ, H*DV).

    The ggml views are q [D, LQ, H, B] (head h at byte offset h*D*es of each
    token row), k [D, LK, HK, B], v [DV, LK, HK, B], dst [DV, H, LQ, B].
    """
    import torch

    lib = load()
    b, lq, hd = q.shape
    _, lk, hkd = k.shape
    d = hd // heads
    dv = v.shape[2] // kv_heads
    if out is None:
        out = torch.empty(b, lq, heads * dv, dtype=torch.float32, device=q.device)
    qs, ks, vs = q.element_size(), k.element_size(), v.element_size()
    dq = describe(q, [d, lq, heads, b], [qs, q.stride(1) * qs, d * qs, q.stride(0) * qs])
    dk = describe(k, [d, lk, kv_heads, b], [ks, k.stride(1) * ks, d * ks, k.stride(0) * ks])
    dvv = describe(v, [dv, lk, kv_heads, b], [vs, v.stride(1) * vs, dv * vs, v.stride(0) * vs])
    do = describe(out, [dv, heads, lq, b], [4, dv * 4, out.stride(1) * 4, out.stride(0) * 4])
    if not lib.sdb_attention_supported(dq, dk, dvv, do):
        raise SdbError(NOT_SUPPORTED, "attention shapes not supported")
    _check(lib.sdb_attention(dq, dk, dvv, do, ctypes.c_float(scale), _chain_ptr(chain),
                             ctypes.c_void_p(_stream_ptr(stream))))
    return out


def group_norm(x, groups: int, eps: float, out=None, chain: Chain | None = None, stream=None):
    """GGML_OP_GROUP_NORM over (N, C, H, W): groups of C/groups (rounded up) channels."""
    import torch

    lib = load()
    if out is None:
        out = torch.empty_like(x)
    _check(lib.sdb_group_norm(describe(x), describe(out), groups, ctypes.c_float(eps), _chain_ptr(chain),
                              ctypes.c_void_p(_stream_ptr(stream))))
    return out


def group_norm_no_alloc(x, groups: int, eps: float, out, chain: Chain | None = None, stream=None):
    """group_norm without any device allocation (sdb_group_norm_no_alloc): out must be given."""
    lib = load()
    _check(lib.sdb_group_norm_no_alloc(describe(x), describe(out), groups, ctypes.c_float(eps), _chain_ptr(chain),
                                       ctypes.c_void_p(_stream_ptr(stream))))
    return out


def norm(x, eps: float, out=None, chain: Chain | None = None, stream=None):
    """GGML_OP_NORM: each row (last torch dimension) to mean 0, variance 1."""
    import torch

    lib = load()
    if out is None:
        out = torch.empty_like(x)
    _check(lib.sdb_norm(describe(x), describe(out), ctypes.c_float(eps), _chain_ptr(chain),
                        ctypes.c_void_p(_stream_ptr(stream))))
    return out


def forget(t_or_ptr, size: int | None = None) -> None:
    """Drops packed weights made from the memory of t (sdasm_forget)."""
    lib = load()
    if size is None:
        ptr, size = t_or_ptr.data_ptr(), t_or_ptr.numel() * t_or_ptr.element_size()
    else:
        ptr = t_or_ptr
    lib.sdb_forget(ctypes.c_void_p(ptr), ctypes.c_size_t(size))
    for a in [a for a in _weights if ptr <= a < ptr + size]:
        del _weights[a]


def store_stats() -> tuple[int, int]:
    lib = load()
    e, b = ctypes.c_int64(), ctypes.c_int64()
    lib.sdb_store_stats(ctypes.byref(e), ctypes.byref(b))
    return e.value, b.value


def set_tuning(spec: str) -> None:
    _check(load().sdb_set_tuning(spec.encode()))


def get_tuning(name: str) -> int:
    v = ctypes.c_int64()
    _check(load().sdb_get_tuning(name.encode(), ctypes.byref(v)))
    return v.value


def device_status(clear: bool = True) -> int:
    return int(load().sdb_device_status(1 if clear else 0))


def launch_count() -> int:
    return int(load().sdb_launch_count())


def token_downsampling(width: int, height: int) -> int:
    return int(load().sdb_token_downsampling(width, height))


# ---------------------------------------------------------------- channels-last images

def describe_nhwc(t) -> Tensor:
    """A contiguous (N, H, W, C) FP32 tensor as the ggml image [W, H, C, N] it holds (channels-last strides)."""
    n, h, w, c = t.shape
    es = t.element_size()
    return describe(t, [w, h, c, n], [c * es, w * c * es, es, h * w * c * es])


def conv2d_nhwc(w, x, stride=(1, 1), padding=(0, 0), dilation=(1, 1), out=None, chain: Chain | None = None,
                stream=None, out_nchw: bool = False):
    """ggml_conv_2d_direct on channels-last images: w (OC, IC, KH, KW), x (N, H, W, IC) -> (N, OH, OW, OC),
    or with out_nchw the output channel-major, (N, OC, OH, OW)."""
    import torch

    lib = load()
    oc, _, kh, kw = w.shape
    n, h, wd, _ = x.shape
    oh = conv_out_size(h, kh, stride[1], padding[1], dilation[1])
    ow = conv_out_size(wd, kw, stride[0], padding[0], dilation[0])
    if out is None:
        shape = (n, oc, oh, ow) if out_nchw else (n, oh, ow, oc)
        out = torch.empty(*shape, dtype=torch.float32, device=x.device)
    params = (ctypes.c_int32 * 6)(stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1])
    _guard_weight(w)
    dy = describe(out) if out_nchw else describe_nhwc(out)
    _check(lib.sdb_conv2d(describe(w), describe_nhwc(x), dy, params, _chain_ptr(chain),
                          ctypes.c_void_p(_stream_ptr(stream))))
    return out


def channel_operand(t):
    """ggml strides of a per-channel operand (C,) for a channels-last image output: broadcast over W, H, N."""
    return [0, 0, 1, 0]


def group_norm_nhwc(x, groups: int, eps: float, out=None, chain: Chain | None = None, stream=None):
    """GGML_OP_GROUP_NORM on a channels-last image (N, H, W, C), C % groups == 0."""
    import torch

    lib = load()
    if out is None:
        out = torch.empty_like(x)
    _check(lib.sdb_group_norm(describe_nhwc(x), describe_nhwc(out), groups, ctypes.c_float(eps), _chain_ptr(chain),
                              ctypes.c_void_p(_stream_ptr(stream))))
    return out


class GroupNormIn:
    """A GroupNorm (+ SiLU) that the next operation applies as it reads its input (sdb_norm_in):
    the statistics of x (group_norm_stats), gamma and beta (C,) or None, groups, SiLU."""

    def __init__(self, stats, groups: int, gamma=None, beta=None, silu: bool = False):
        self.stats, self.groups, self.gamma, self.beta, self.silu = stats, groups, gamma, beta, silu
        self.c = NormIn(stats.data_ptr(), gamma.data_ptr() if gamma is not None else None,
                        beta.data_ptr() if beta is not None else None, groups, 1 if silu else 0)


def group_norm_stats(x, groups: int, eps: float, out=None, stream=None):
    """Mean and 1 / sqrt(variance + eps) per image and group of a channels-last image (N, H, W, C):
    (N, groups, 2) FP32 (sdb_group_norm_stats)."""
    import torch

    lib = load()
    if out is None:
        out = torch.empty(x.shape[0], groups, 2, dtype=torch.float32, device=x.device)
    _check(lib.sdb_group_norm_stats(describe_nhwc(x), groups, ctypes.c_float(eps), ctypes.c_void_p(out.data_ptr()),
                                    ctypes.c_void_p(_stream_ptr(stream))))
    return out


def conv2d_nhwc_normed(w, x, norm: GroupNormIn, stride=(1, 1), padding=(0, 0), dilation=(1, 1), out=None,
                       chain: Chain | None = None, stream=None):
    """conv2d_nhwc of GroupNorm(x) [+ SiLU], the normalisation applied as the convolution reads x."""
    import torch

    lib = load()
    oc, _, kh, kw = w.shape
    n, h, wd, _ = x.shape
    oh = conv_out_size(h, kh, stride[1], padding[1], dilation[1])
    ow = conv_out_size(wd, kw, stride[0], padding[0], dilation[0])
    if out is None:
        out = torch.empty(n, oh, ow, oc, dtype=torch.float32, device=x.device)
    params = (ctypes.c_int32 * 6)(stride[0], stride[1], padding[0], padding[1], dilation[0], dilation[1])
    _guard_weight(w)
    _check(lib.sdb_conv2d_normed(describe(w), describe_nhwc(x), describe_nhwc(out), params, ctypes.byref(norm.c),
                                 _chain_ptr(chain), ctypes.c_void_p(_stream_ptr(stream))))
    return out


def mul_mat_normed(w, x, norm: GroupNormIn, out=None, chain: Chain | None = None, stream=None):
    """mul_mat of GroupNorm(x) [+ SiLU]: x (N, P, C), the P positions of each of N images."""
    import torch

    lib = load()
    if out is None:
        out = torch.empty(*x.shape[:-1], w.shape[0], dtype=torch.float32, device=x.device)
    _guard_weight(w)
    _check(lib.sdb_mul_mat_normed(describe(w), describe(x), describe(out), ctypes.byref(norm.c), _chain_ptr(chain),
                                  ctypes.c_void_p(_stream_ptr(stream))))
    return out


def mul_mat_layer_normed(w, x, eps: float, norm_chain: Chain | None = None, out=None, chain: Chain | None = None,
                         gated: bool = False, stream=None):
    """mul_mat (or mul_mat_gated) of LayerNorm(x) with its chain (gamma, beta), the normalisation done in
    the linear layer's split of the rows: x (..., K) -> (..., N) (N / 2 gated)."""
    import torch

    lib = load()
    if out is None:
        n = w.shape[0] // 2 if gated else w.shape[0]
        out = torch.empty(*x.shape[:-1], n, dtype=torch.float32, device=x.device)
    _guard_weight(w)
    fn = lib.sdb_mul_mat_gated_layer_normed if gated else lib.sdb_mul_mat_layer_normed
    _check(fn(describe(w), describe(x), describe(out), ctypes.c_float(eps), _chain_ptr(norm_chain), _chain_ptr(chain),
              ctypes.c_void_p(_stream_ptr(stream))))
    return out


def concat_channels_nhwc(a, b, out=None, stream=None):
    """GGML_OP_CONCAT along C of channels-last images (N, H, W, Ca) and (N, H, W, Cb)."""
    import torch

    lib = load()
    if out is None:
        out = torch.empty(*a.shape[:3], a.shape[3] + b.shape[3], dtype=torch.float32, device=a.device)
    _check(lib.sdb_concat(describe_nhwc(a), describe_nhwc(b), describe_nhwc(out), 2,
                          ctypes.c_void_p(_stream_ptr(stream))))
    return out


def upscale_nearest_nhwc(x, factor: int = 2, out=None, stream=None):
    """GGML_OP_UPSCALE (nearest) of a channels-last image by an integer factor."""
    import torch

    lib = load()
    n, h, w, c = x.shape
    if out is None:
        out = torch.empty(n, h * factor, w * factor, c, dtype=torch.float32, device=x.device)
    _check(lib.sdb_upscale_nearest(describe_nhwc(x), describe_nhwc(out), ctypes.c_void_p(_stream_ptr(stream))))
    return out


def coarser_tokens(x, width: int, height: int, factor: int, out=None, stream=None):
    """ToDo's keys' and values' tokens: x (N, height * width, C) tokens of a grid, row after row ->
    (N, ceil(height / f) * ceil(width / f), C), every f-th token of every f-th row."""
    import torch

    lib = load()
    n, l, c = x.shape
    if l != width * height:
        raise SdbError(INVALID, "coarser_tokens: the tokens are not the grid's")
    w2, h2 = -(-width // factor), -(-height // factor)
    if out is None:
        out = torch.empty(n, h2 * w2, c, dtype=torch.float32, device=x.device)
    s = [v * 4 for v in x.stride()]
    src = describe(x, [c, width, height, n], [s[2], s[1], s[1] * width, s[0]])
    dst = describe(out, [c, w2, h2, n], [4, 4 * c, 4 * c * w2, 4 * c * w2 * h2])
    _check(lib.sdb_coarser_tokens(src, dst, factor, ctypes.c_void_p(_stream_ptr(stream))))
    return out


def timestep_embedding(t, dim: int, max_period: int = 10000, out=None, stream=None):
    """GGML_OP_TIMESTEP_EMBEDDING: t (N,) FP32 -> (N, dim) = [cos(t f) | sin(t f)]."""
    import torch

    lib = load()
    if out is None:
        out = torch.empty(t.shape[0], dim, dtype=torch.float32, device=t.device)
    _check(lib.sdb_timestep_embedding(describe(t), describe(out), dim, max_period,
                                      ctypes.c_void_p(_stream_ptr(stream))))
    return out


def euler_ancestral_cfg_step(eps, x, x_in, noise, cfg: float, sigma: float, sigma_next: float, c_in_next: float,
                             stream=None):
    """The ancestral Euler step with guidance: x += (sigma_down - sigma) e + sigma_up noise (see sdb.h)."""
    lib = load()
    _check(lib.sdb_euler_ancestral_cfg_step(ctypes.c_void_p(eps.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                            ctypes.c_void_p(x_in.data_ptr() if x_in is not None else 0),
                                            ctypes.c_void_p(noise.data_ptr()), ctypes.c_int64(x.numel()),
                                            ctypes.c_float(cfg), ctypes.c_float(sigma), ctypes.c_float(sigma_next),
                                            ctypes.c_float(c_in_next), ctypes.c_void_p(_stream_ptr(stream))))


def euler_cfg_step(eps, x, x_in, cfg: float, sigma: float, sigma_next: float, c_in_next: float, stream=None):
    """x += (sigma_next - sigma) (eps_u + cfg (eps_c - eps_u)); x_in[0] = x_in[1] = x c_in_next (eps = [eps_u, eps_c])."""
    lib = load()
    _check(lib.sdb_euler_cfg_step(ctypes.c_void_p(eps.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                                  ctypes.c_void_p(x_in.data_ptr() if x_in is not None else 0),
                                  ctypes.c_int64(x.numel()), ctypes.c_float(cfg), ctypes.c_float(sigma),
                                  ctypes.c_float(sigma_next), ctypes.c_float(c_in_next),
                                  ctypes.c_void_p(_stream_ptr(stream))))
