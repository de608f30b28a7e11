"""A small stand-in for ggml, for testing the sdasm.h hook surface without ggml.

ggml and stable-diffusion.cpp are not in this repository.  This module builds
ggml graphs out of the struct layout of include/ggml_mirror.h (the operation
numbers are read from that header), with ggml's semantics for what the tests
need: new tensors, views and reshapes, in-place and out-of-place ADD and MUL
with broadcasting, DUP, CONT, the unary SiLU/GELU, SCALE, and the operations the
hooks take (MUL_MAT, CONV_2D, FLASH_ATTN_EXT, GROUP_NORM, NORM).  The graph's
node order is ggml_build_forward_expand's: a depth-first walk over the sources,
left to right, a node after its sources, tensors without an operation as leaves.

`run()` is ggml's patched graph loop (patches/ggml/0003): for each node it asks
sdasm_compute_nodes() first and skips the nodes it reports as computed;
otherwise it computes the node itself (numpy for host memory, torch for device
memory), as ggml's CPU kernels would.  The hooks see the same structs either way.

Tensors live in host memory (numpy buffers: the stock CPU backend, which the
hooks stage through the device) or, with `Graph("cuda")`, in device memory
(torch CUDA tensors, which the kernels read in place).
"""
from __future__ import annotations

import ctypes
import math
import re
from pathlib import Path

import numpy as np

import oracle

ROOT = Path(__file__).resolve().parent.parent
MIRROR = ROOT / "include" / "ggml_mirror.h"


def _ops() -> dict[str, int]:
    text = MIRROR.read_text()
    body = re.search(r"#define SDB_GGML_OPS\(X\)(.*?)\n\n", text, re.S).group(1)
    names = re.findall(r"X\((\w+)\)", body)
    return {n: i for i, n in enumerate(names)}


OP = _ops()
TYPE_F32, TYPE_F16 = 0, 1
UNARY_SILU, UNARY_GELU = 0, 1
FLAG_OUTPUT, FLAG_COMPUTE = 2, 16


class GgmlTensor(ctypes.Structure):
    pass


GgmlTensor._fields_ = [
    ("type", ctypes.c_int), ("buffer", ctypes.c_void_p), ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_size_t * 4),
    ("op", ctypes.c_int), ("op_params", ctypes.c_int32 * 16), ("flags", ctypes.c_int32),
    ("src", ctypes.POINTER(GgmlTensor) * 10), ("view_src", ctypes.POINTER(GgmlTensor)), ("view_offs", ctypes.c_size_t),
    ("data", ctypes.c_void_p), ("name", ctypes.c_char * 64), ("extra", ctypes.c_void_p), ("padding", ctypes.c_char * 8),
]


class ComputeParams(ctypes.Structure):
    _fields_ = [("ith", ctypes.c_int), ("nth", ctypes.c_int), ("wsize", ctypes.c_size_t), ("wdata", ctypes.c_void_p),
                ("threadpool", ctypes.c_void_p), ("use_ref", ctypes.c_bool)]


def _f32_bits(x: float) -> int:
    return int(np.array([x], dtype=np.float32).view(np.int32)[0])


class Tensor:
    """A ggml tensor: the ctypes struct, its sources, and the memory it views."""

    def __init__(self, graph: "Graph", ttype: int, ne, nb, base, offset: int, op: int = 0, srcs=(), params=(),
                 view_src: "Tensor | None" = None):
        self.graph = graph
        self.s = GgmlTensor()
        self.s.type = ttype
        for k in range(4):
            self.s.ne[k] = int(ne[k])
            self.s.nb[k] = int(nb[k])
        self.s.op = op
        for i, p in enumerate(params):
            self.s.op_params[i] = p
        self.srcs = list(srcs)
        for i, t in enumerate(self.srcs):
            if t is not None:
                self.s.src[i] = ctypes.pointer(t.s)
        self.view_src = view_src
        if view_src is not None:
            self.s.view_src = ctypes.pointer(view_src.s)
        self.base = base          # the buffer (numpy uint8 array or torch uint8 tensor)
        self.offset = offset      # bytes into it
        self.s.data = graph.address(base) + offset
        self.s.flags = FLAG_COMPUTE if op != OP["NONE"] else 0

    @property
    def ne(self):
        return [self.s.ne[k] for k in range(4)]

    @property
    def nb(self):
        return [self.s.nb[k] for k in range(4)]

    @property
    def esize(self):
        return 4 if self.s.type == TYPE_F32 else 2

    def array(self):
        """The elements, [ne3, ne2, ne1, ne0], as a strided view of the memory."""
        return self.graph.view(self)

    def numpy(self) -> np.ndarray:
        a = self.array()
        return a.detach().cpu().numpy().copy() if hasattr(a, "detach") else np.array(a)


class Graph:
    """A ggml context and graph; device "host" (numpy) or "cuda" (torch)."""

    def __init__(self, device: str = "host"):
        self.device = device
        self.tensors: list[Tensor] = []
        self.buffers: list = []

    def release(self, lib):
        """Frees the context's buffers as ggml does: sdasm_forget() on each first (patch 0004),
        so that nothing kept from them outlives their memory."""
        for b in self.buffers:
            n = b.nbytes if isinstance(b, np.ndarray) else b.numel()
            lib.sdasm_forget.restype = None
            lib.sdasm_forget.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
            lib.sdasm_forget(ctypes.c_void_p(self.address(b)), ctypes.c_size_t(n))
        self.buffers.clear()

    # ------------------------------------------------ memory
    def buffer(self, nbytes: int):
        if self.device == "host":
            raw = np.zeros(nbytes + 128, dtype=np.uint8)
            skip = (-raw.ctypes.data) % 64
            b = raw[skip:skip + nbytes]
        else:
            import torch

            b = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=self.device)
        self.buffers.append(b)
        return b

    def address(self, base) -> int:
        return base.ctypes.data if isinstance(base, np.ndarray) else base.data_ptr()

    def view(self, t: Tensor):
        dtype_np = np.float32 if t.s.type == TYPE_F32 else np.float16
        shape = tuple(reversed(t.ne))
        if isinstance(t.base, np.ndarray):
            flat = t.base.view(dtype_np) if t.offset % t.esize == 0 else None
            return np.lib.stride_tricks.as_strided(flat[t.offset // t.esize:], shape=shape,
                                                   strides=tuple(reversed(t.nb)))
        import torch

        flat = t.base.view(torch.float32 if t.s.type == TYPE_F32 else torch.float16)
        return torch.as_strided(flat, shape, tuple(n // t.esize for n in reversed(t.nb)), t.offset // t.esize)

    def fill(self, t: Tensor, values: np.ndarray):
        v = np.asarray(values, dtype=np.float32 if t.s.type == TYPE_F32 else np.float16).reshape(
            tuple(reversed(t.ne)))
        a = self.view(t)
        if isinstance(a, np.ndarray):
            a[...] = v
        else:
            import torch

            a.copy_(torch.from_numpy(v).to(a.device))

    def _add(self, t: Tensor) -> Tensor:
        self.tensors.append(t)
        return t

    @staticmethod
    def _dense_nb(ne, es):
        nb = [es]
        for k in range(1, 4):
            nb.append(nb[-1] * ne[k - 1])
        return nb

    def _new(self, ttype, ne, op=0, srcs=(), params=()) -> Tensor:
        ne = list(ne) + [1] * (4 - len(ne))
        es = 4 if ttype == TYPE_F32 else 2
        nb = self._dense_nb(ne, es)
        base = self.buffer(int(np.prod(ne)) * es)
        return self._add(Tensor(self, ttype, ne, nb, base, 0, op, srcs, params))

    @staticmethod
    def _root(a: Tensor) -> Tensor:
        """ggml points a view of a view at the tensor that owns the memory."""
        return a.view_src if a.view_src is not None else a

    def _view_of(self, a: Tensor, ne, nb, offset, op) -> Tensor:
        return self._add(Tensor(self, a.s.type, ne, nb, a.base, a.offset + offset, op, [a],
                                view_src=self._root(a)))

    # ------------------------------------------------ leaves
    def new_f32(self, ne, fill: float | None = None, rng=None) -> Tensor:
        t = self._new(TYPE_F32, ne)
        if fill is not None:
            self.fill(t, oracle.uniform(rng or oracle.generator(), tuple(reversed(t.ne)), fill))
        return t

    def new_f16(self, ne, fill: float | None = None, rng=None) -> Tensor:
        t = self._new(TYPE_F16, ne)
        if fill is not None:
            self.fill(t, oracle.uniform(rng or oracle.generator(), tuple(reversed(t.ne)), fill, np.float16))
        return t

    # ------------------------------------------------ views
    def reshape_4d(self, a: Tensor, *ne) -> Tensor:
        return self._view_of(a, ne, self._dense_nb(ne, a.esize), 0, OP["RESHAPE"])

    def view_2d(self, a: Tensor, ne0, ne1, nb1, offset) -> Tensor:
        return self._view_of(a, [ne0, ne1, 1, 1], [a.esize, nb1, nb1 * ne1, nb1 * ne1], offset, OP["VIEW"])

    def view_4d(self, a: Tensor, ne, nb, offset) -> Tensor:
        return self._view_of(a, ne, nb, offset, OP["VIEW"])

    # ------------------------------------------------ operations
    def _inplace(self, a: Tensor, op, srcs, params=()) -> Tensor:
        return self._add(Tensor(self, a.s.type, a.ne, a.nb, a.base, a.offset, op, srcs, params,
                                view_src=self._root(a)))

    def add(self, a, b):
        return self._new(TYPE_F32, a.ne, OP["ADD"], [a, b])

    def add_inplace(self, a, b):
        return self._inplace(a, OP["ADD"], [a, b])

    def mul(self, a, b):
        return self._new(TYPE_F32, a.ne, OP["MUL"], [a, b])

    def mul_inplace(self, a, b):
        return self._inplace(a, OP["MUL"], [a, b])

    def silu_inplace(self, a):
        return self._inplace(a, OP["UNARY"], [a], [UNARY_SILU])

    def gelu_inplace(self, a):
        return self._inplace(a, OP["UNARY"], [a], [UNARY_GELU])

    def scale(self, a, s: float):
        return self._new(TYPE_F32, a.ne, OP["SCALE"], [a], [_f32_bits(s)])

    def dup(self, a):
        return self._new(a.s.type, a.ne, OP["DUP"], [a])

    def cont(self, a):
        return self._new(a.s.type, a.ne, OP["CONT"], [a])

    def mul_mat(self, w, x):
        return self._new(TYPE_F32, [w.ne[1], x.ne[1], x.ne[2], x.ne[3]], OP["MUL_MAT"], [w, x])

    def conv_2d_direct(self, w, x, s0, s1, p0, p1, d0, d1):
        ow = (x.ne[0] + 2 * p0 - d0 * (w.ne[0] - 1) - 1) // s0 + 1
        oh = (x.ne[1] + 2 * p1 - d1 * (w.ne[1] - 1) - 1) // s1 + 1
        return self._new(TYPE_F32, [ow, oh, w.ne[3], x.ne[3]], OP["CONV_2D"], [w, x], [s0, s1, p0, p1, d0, d1])

    def flash_attn_ext(self, q, k, v, scale: float):
        return self._new(TYPE_F32, [v.ne[0], q.ne[2], q.ne[1], q.ne[3]], OP["FLASH_ATTN_EXT"], [q, k, v],
                         [_f32_bits(scale), 0, 0])

    def group_norm(self, a, groups: int, eps: float):
        return self._new(TYPE_F32, a.ne, OP["GROUP_NORM"], [a], [groups, _f32_bits(eps)])

    def norm(self, a, eps: float):
        return self._new(TYPE_F32, a.ne, OP["NORM"], [a], [_f32_bits(eps)])

    # ------------------------------------------------ the graph
    def build(self, out: Tensor) -> list[Tensor]:
        """ggml_build_forward_expand's node order (sources first, left to right)."""
        order: list[Tensor] = []
        seen: set[int] = set()

        def visit(t: Tensor):
            if id(t) in seen:
                return
            seen.add(id(t))
            for s in t.srcs:
                if s is not None:
                    visit(s)
            if t.s.op != OP["NONE"]:
                order.append(t)

        visit(out)
        out.s.flags |= FLAG_OUTPUT
        return order


def node_array(nodes: list[Tensor]):
    arr = (ctypes.POINTER(GgmlTensor) * len(nodes))()
    for i, t in enumerate(nodes):
        arr[i] = ctypes.pointer(t.s)
    return arr


def compute_nodes(lib, nodes: list[Tensor], index: int, ith: int = 0, nth: int = 1) -> int:
    params = ComputeParams(ith, nth, 0, None, None, False)
    lib.sdasm_compute_nodes.restype = ctypes.c_int
    lib.sdasm_compute_nodes.argtypes = [ctypes.POINTER(ComputeParams), ctypes.POINTER(ctypes.POINTER(GgmlTensor)),
                                        ctypes.c_int, ctypes.c_int]
    return lib.sdasm_compute_nodes(ctypes.byref(params), node_array(nodes), len(nodes), index)


# ---------------------------------------------------------------- ggml's own kernels, for nodes not taken

def _torch_or_np(a):
    return "torch" if hasattr(a, "detach") else "np"


def _silu(x):
    if _torch_or_np(x) == "np":
        return oracle.silu(x)
    import torch

    return torch.from_numpy(oracle.silu(x.detach().cpu().numpy())).to(x.device)


def _gelu(x):
    if _torch_or_np(x) == "np":
        return oracle.gelu(x)
    import torch

    return torch.from_numpy(oracle.gelu(x.detach().cpu().numpy())).to(x.device)


def compute_by_ggml(t: Tensor):
    """One node computed as ggml's CPU kernels would (the element-wise nodes the tests use)."""
    op = t.s.op
    if op in (OP["RESHAPE"], OP["VIEW"], OP["PERMUTE"], OP["TRANSPOSE"], OP["NONE"]):
        return
    dst = t.array()
    a = t.srcs[0].array()
    if op in (OP["DUP"], OP["CONT"]):
        dst[...] = a
    elif op == OP["ADD"]:
        dst[...] = a + t.srcs[1].array()
    elif op == OP["MUL"]:
        dst[...] = a * t.srcs[1].array()
    elif op == OP["UNARY"]:
        f = _silu if t.s.op_params[0] == UNARY_SILU else _gelu
        dst[...] = f(a)
    elif op == OP["SCALE"]:
        dst[...] = a * np.float32(np.array([t.s.op_params[0]], dtype=np.int32).view(np.float32)[0])
    else:
        raise NotImplementedError(f"the hooks were expected to take op {op}")


def run(lib, nodes: list[Tensor]) -> list[int]:
    """ggml's patched graph loop (patch 0003): the counts sdasm_compute_nodes returned, node by node."""
    counts = []
    i = 0
    while i < len(nodes):
        n = compute_nodes(lib, nodes, i)
        counts.append(n)
        if n > 0:
            i += n
        else:
            compute_by_ggml(nodes[i])
            i += 1
    if nodes and nodes[0].graph.device != "host":
        import torch

        torch.cuda.synchronize()
    return counts


def forget(lib, t: Tensor):
    """What ggml's buffer writes call (patch 0004) before a tensor's data changes."""
    lib.sdasm_forget.restype = None
    lib.sdasm_forget.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    nbytes = t.esize + sum((t.ne[k] - 1) * t.nb[k] for k in range(4))
    lib.sdasm_forget(ctypes.c_void_p(t.s.data), ctypes.c_size_t(nbytes))


def scale_of_head(d: int) -> float:
    return 1.0 / math.sqrt(d)
