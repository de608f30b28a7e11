"""The sdasm.h hook surface (include/sdasm.h, csrc/hooks.cu) through the C ABI, on ggml graphs.

The graphs are ops_test's fusion cases (tests/ops_test.cc:953-1117 of the
reference) built as ggml tensors of include/ggml_mirror.h's layout
(tests/ggml_graph.py), run by ggml's patched graph loop: sdasm_compute_nodes()
is offered every node and reports how many it computed.  Checked, as the
reference's ops_test checks them:
  * the node counts: the operation with its chain (bias, scale, residual in
    place, not in place, in the residual's own memory, the GEGLU pattern);
  * fused against apart (tuning fuse=0, every element-wise node left to ggml)
    within 1e-6 of the largest output (ops_test.cc:591-631);
  * the result against the float64 exact oracle (ops_test metric, or 1e-6 of
    the largest output for the normalisations, whose form is the reference's);
  * sdasm_forget(): weights set anew are used, and without it the device copy
    is kept (ops_test.cc:643-719, the store cases);
  * threads other than 0 return the same count without computing.
Tensors live in host memory (the stock CPU backend's buffers, staged through
the device per node) and, for two graphs, in device memory.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

import ggml_graph as gg
import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(cuda):
    import sdb

    return sdb.load()


def tuning(fuse: int):
    import sdb

    sdb.set_tuning(f"fuse={fuse}")


# ---------------------------------------------------------------- ops_test's fusion graphs
# Each builder returns (the output tensor; exact(), which gives (exact, magnitude, bound) or, for
# a normalisation, the reference's single-precision result; the node counts sdasm_compute_nodes
# returns with fuse=1, one per offered node that it did not take (0) or took (> 0)).

def conv_exact(w, x, pad, steps):
    """Exact convolution (ops_test.cc:385-424) with the chain's additions and multiplications in
    float64, and the bound: 1e-6, or for a 3x3 kernel (which Winograd's F(4x4) may take) at most
    1.5x the reference's own single-precision F(4x4) form's error (tests/test_winograd_gpu.py)."""
    wn, xn = w.numpy(), x.numpy()
    ex, mag = oracle.conv2d_exact(wn, xn, (1, 1), pad, (1, 1))
    bound = oracle.K_B200
    if wn.shape[2:] == (3, 3):
        bound = max(bound, 1.5 * oracle.metric(oracle.winograd_f32(wn, xn, pad, 4), ex, mag))
    for kind, t in steps:
        o = t.numpy().astype(np.float64)
        if kind == "add":
            ex, mag = ex + o, mag + np.abs(o)
        else:
            ex, mag = ex * o, mag * np.abs(o)
    return ex, mag, bound


def linear_exact(w, x, steps):
    ex, mag = oracle.mul_mat_exact(w.numpy()[0, 0], x.numpy())
    for kind, t in steps:
        o = t.numpy().astype(np.float64)
        if o.ndim == 4 and ex.ndim == 3:
            o = o.reshape(o.shape[1:]) if o.shape[0] == 1 else o
        ex, mag = ex + o, mag + np.abs(o)
    return ex, mag, oracle.K_B200


def case_conv_bias(g, r):
    w = g.new_f16([3, 3, 24, 40], 0.25, r)
    x = g.new_f32([40, 36, 24, 2], 1.0, r)
    b = g.new_f32([40], 1.0, r)
    y = g.conv_2d_direct(w, x, 1, 1, 1, 1, 1, 1)
    out = g.add_inplace(y, g.reshape_4d(b, 1, 1, 40, 1))
    return out, lambda: conv_exact(w, x, (1, 1), [("add", g.reshape_4d(b, 1, 1, 40, 1))]), [3]


def case_conv1x1_bias_scale(g, r):
    w = g.new_f16([1, 1, 16, 20], 0.25, r)
    x = g.new_f32([17, 9, 16, 2], 1.0, r)
    b = g.new_f32([20], 1.0, r)
    e = g.new_f32([1, 1, 20, 2], 1.0, r)
    y = g.conv_2d_direct(w, x, 1, 1, 0, 0, 1, 1)
    bb = g.reshape_4d(b, 1, 1, 20, 1)
    y = g.add_inplace(y, bb)
    out = g.mul_inplace(y, e)
    return out, lambda: conv_exact(w, x, (0, 0), [("add", bb), ("mul", e)]), [4]


def case_winograd_bias_residual(g, r):
    w = g.new_f16([3, 3, 16, 24], 0.25, r)
    x = g.new_f32([66, 40, 16, 1], 1.0, r)
    b = g.new_f32([24], 1.0, r)
    res = g.new_f32([66, 40, 24, 1], 1.0, r)
    y = g.conv_2d_direct(w, x, 1, 1, 1, 1, 1, 1)
    bb = g.reshape_4d(b, 1, 1, 24, 1)
    y = g.add_inplace(y, bb)
    out = g.add_inplace(y, res)
    return out, lambda: conv_exact(w, x, (1, 1), [("add", bb), ("add", res)]), [4]


def case_conv_bias_residual_apart(g, r):
    w = g.new_f16([3, 3, 24, 40], 0.25, r)
    x = g.new_f32([40, 36, 24, 2], 1.0, r)
    b = g.new_f32([40], 1.0, r)
    res = g.new_f32([40, 36, 40, 2], 1.0, r)
    y = g.conv_2d_direct(w, x, 1, 1, 1, 1, 1, 1)
    bb = g.reshape_4d(b, 1, 1, 40, 1)
    y = g.add_inplace(y, bb)
    out = g.add(y, res)
    return out, lambda: conv_exact(w, x, (1, 1), [("add", bb), ("add", res)]), [4]


def case_small_winograd_residual_left(g, r):
    w = g.new_f16([3, 3, 64, 48], 0.25, r)
    x = g.new_f32([16, 16, 64, 2], 1.0, r)
    res = g.new_f32([16, 16, 48, 2], 1.0, r)
    out = g.add(res, g.conv_2d_direct(w, x, 1, 1, 1, 1, 1, 1))
    return out, lambda: conv_exact(w, x, (1, 1), [("add", res)]), [2]


def case_linear_bias_residual_apart(g, r):
    w = g.new_f16([96, 70], 0.25, r)
    x = g.new_f32([96, 50, 2], 1.0, r)
    b = g.new_f32([70], 1.0, r)
    res = g.new_f32([70, 50, 2], 1.0, r)
    out = g.add(g.add_inplace(g.mul_mat(w, x), b), res)
    return out, lambda: linear_exact(w, x, [("add", b), ("add", res)]), [3]


def case_conv_bias_residual_own(g, r):
    w = g.new_f16([1, 1, 96, 40], 0.25, r)
    x = g.new_f32([40, 36, 96, 2], 1.0, r)
    b = g.new_f32([40], 1.0, r)
    res = g.new_f32([40, 36, 40, 2], 1.0, r)
    y = g.conv_2d_direct(w, x, 1, 1, 0, 0, 1, 1)
    bb = g.reshape_4d(b, 1, 1, 40, 1)
    y = g.add_inplace(y, bb)
    out = g.add_inplace(g.dup(res), y)
    return out, lambda: conv_exact(w, x, (0, 0), [("add", bb), ("add", res)]), [0, 4]


def case_winograd_residual_own(g, r):
    w = g.new_f16([3, 3, 16, 24], 0.25, r)
    x = g.new_f32([66, 40, 16, 1], 1.0, r)
    b = g.new_f32([24], 1.0, r)
    res = g.new_f32([66, 40, 24, 1], 1.0, r)
    y = g.conv_2d_direct(w, x, 1, 1, 1, 1, 1, 1)
    bb = g.reshape_4d(b, 1, 1, 24, 1)
    y = g.add_inplace(y, bb)
    out = g.add_inplace(g.dup(res), y)
    return out, lambda: conv_exact(w, x, (1, 1), [("add", bb), ("add", res)]), [0, 4]


def case_small_winograd_residual_own(g, r):
    w = g.new_f16([3, 3, 64, 48], 0.25, r)
    x = g.new_f32([15, 9, 64, 2], 1.0, r)
    res = g.new_f32([15, 9, 48, 2], 1.0, r)
    out = g.add_inplace(g.dup(res), g.conv_2d_direct(w, x, 1, 1, 1, 1, 1, 1))
    return out, lambda: conv_exact(w, x, (1, 1), [("add", res)]), [0, 2]


def case_linear_bias_residual_own(g, r):
    w = g.new_f16([300, 70], 0.25, r)
    x = g.new_f32([300, 1100, 2], 1.0, r)
    b = g.new_f32([70], 1.0, r)
    res = g.new_f32([70, 1100, 2], 1.0, r)
    out = g.add_inplace(g.dup(res), g.add_inplace(g.mul_mat(w, x), b))
    return out, lambda: linear_exact(w, x, [("add", b), ("add", res)]), [0, 3]


def case_linear_bias(g, r):
    w = g.new_f16([96, 70], 0.25, r)
    x = g.new_f32([96, 50, 2], 1.0, r)
    b = g.new_f32([70], 1.0, r)
    out = g.add_inplace(g.mul_mat(w, x), b)
    return out, lambda: linear_exact(w, x, [("add", b)]), [2]


def norm_reference(kind, x, groups, eps, steps):
    x64 = x.numpy()
    y = oracle.group_norm_ref(x64[...], groups, eps) if kind == "group" else oracle.norm_ref(x64, eps)
    return oracle.apply_chain(y, [(k, t.numpy() if t is not None else None) for k, t in steps])


def case_group_norm_silu(g, r):
    x = g.new_f32([36, 20, 64, 2], 3.0, r)
    gm = g.new_f32([1, 1, 64, 1], 1.0, r)
    bt = g.new_f32([1, 1, 64, 1], 1.0, r)
    y = g.group_norm(x, 32, 1e-6)
    y = g.mul_inplace(y, gm)
    y = g.add_inplace(y, bt)
    out = g.silu_inplace(y)
    return out, lambda: norm_reference("group", x, 32, 1e-6, [("mul", gm), ("add", bt), ("silu", None)]), [4]


def case_group_norm_ragged(g, r):
    x = g.new_f32([13, 7, 30, 1], 3.0, r)
    gm = g.new_f32([1, 1, 30, 1], 1.0, r)
    bt = g.new_f32([1, 1, 30, 1], 1.0, r)
    y = g.group_norm(x, 10, 1e-5)
    y = g.mul_inplace(y, gm)
    y = g.add_inplace(y, bt)
    out = g.silu_inplace(y)
    return out, lambda: norm_reference("group", x, 10, 1e-5, [("mul", gm), ("add", bt), ("silu", None)]), [4]


def case_layer_norm(g, r):
    x = g.new_f32([320, 77, 2], 3.0, r)
    gm = g.new_f32([320], 1.0, r)
    bt = g.new_f32([320], 1.0, r)
    y = g.norm(x, 1e-5)
    y = g.mul_inplace(y, gm)
    out = g.add_inplace(y, bt)
    return out, lambda: norm_reference("layer", x, 0, 1e-5, [("mul", gm), ("add", bt)]), [3]


def case_geglu(g, r):
    """stable-diffusion.cpp's GEGLU: the linear layer, its bias, two half views, the gate
    made contiguous, its GELU in place and the product (fusion.cc:347-394)."""
    w = g.new_f16([320, 2 * 160], 0.25, r)
    x = g.new_f32([320, 77, 2], 1.0, r)
    b = g.new_f32([2 * 160], 1.0, r)
    y = g.add_inplace(g.mul_mat(w, x), b)
    half = 160
    xin = g.view_4d(y, [half, 77, 2, 1], [4, y.nb[1], y.nb[2], y.nb[3]], 0)
    gate = g.view_4d(y, [half, 77, 2, 1], [4, y.nb[1], y.nb[2], y.nb[3]], half * 4)
    gate = g.gelu_inplace(g.cont(gate))
    out = g.mul(xin, gate)

    def exact():
        ex, mag = oracle.gated_exact(w.numpy()[0, 0], x.numpy()[0], b.numpy().reshape(-1))
        return ex, mag, oracle.K_B200

    return out, exact, [7]


CASES = {
    "conv2d, bias": case_conv_bias,
    "conv2d 1x1, bias, scale per image": case_conv1x1_bias_scale,
    "conv2d by Winograd, bias, residual": case_winograd_bias_residual,
    "conv2d, bias, residual not in place": case_conv_bias_residual_apart,
    "conv2d of small images by Winograd, residual on the left": case_small_winograd_residual_left,
    "linear, bias, residual not in place": case_linear_bias_residual_apart,
    "conv2d, bias, residual in its own memory": case_conv_bias_residual_own,
    "conv2d by Winograd, residual in its own memory": case_winograd_residual_own,
    "conv2d of small images by Winograd, residual in its own memory": case_small_winograd_residual_own,
    "linear, bias, residual in its own memory": case_linear_bias_residual_own,
    "linear, bias": case_linear_bias,
    "group norm, scale, shift, SiLU": case_group_norm_silu,
    "group norm of rows of no multiple of eight, scale, shift": case_group_norm_ragged,
    "layer norm, scale, shift": case_layer_norm,
    "GEGLU (linear, bias, gated GELU)": case_geglu,
}


def run_graph(lib, builder, device, fuse):
    """Builds the graph afresh (the residual copies are remade by each computation) and runs it."""
    tuning(fuse)
    g = gg.Graph(device)
    try:
        out, exact, counts = builder(g, oracle.generator(oracle.SEED))
        nodes = g.build(out)
        got = gg.run(lib, nodes)
        result = out.numpy()
        # The float64 check reads the inputs after the graph is released: copy them now.
        r = exact()
        return result, (lambda: r), counts, got, len(nodes)
    finally:
        g.release(lib)
        tuning(1)


@pytest.mark.parametrize("name", list(CASES))
def test_fusion_graph_through_the_hooks(lib, name):
    fused, exact, counts, got, n = run_graph(lib, CASES[name], "host", 1)
    assert got == counts, f"node counts {got}, expected {counts}"
    apart, _, _, got_apart, _ = run_graph(lib, CASES[name], "host", 0)
    assert sum(c for c in got_apart if c > 0) == sum(1 for c in got_apart if c > 0), got_apart  # heads only
    assert np.all(np.isfinite(fused))
    largest = np.abs(apart).max()
    assert np.abs(fused.astype(np.float64) - apart).max() <= oracle.K_FUSED_APART * largest
    r = exact()
    if isinstance(r, tuple):
        ex, mag, bound = r
        assert oracle.metric(fused.reshape(ex.shape), ex, mag) <= bound
    else:
        assert np.abs(fused - r).max() <= 1e-6 * np.abs(r).max()


@pytest.mark.parametrize("name", ["linear, bias, residual in its own memory", "GEGLU (linear, bias, gated GELU)",
                                  "conv2d, bias, residual not in place"])
def test_fusion_graph_in_device_memory(lib, name):
    """ggml buffers in device memory: the kernels read and write them in place."""
    fused, exact, counts, got, _ = run_graph(lib, CASES[name], "cuda", 1)
    assert got == counts
    ex, mag, bound = exact()
    assert oracle.metric(fused.reshape(ex.shape), ex, mag) <= bound


def test_attention_node(lib):
    """FLASH_ATTN_EXT of permuted q/k/v views, as stable-diffusion.cpp builds it (sd.cpp patch 0002)."""
    d, lq, lk, h, b = 40, 150, 77, 2, 2
    g = gg.Graph("host")
    r = oracle.generator(oracle.SEED)
    qd = g.new_f32([d, h, lq, b], 1.0, r)   # [B, LQ, H*D] rows, viewed as [D, LQ, H, B]
    kd = g.new_f32([d, h, lk, b], 1.0, r)
    vd = g.new_f32([d, h, lk, b], 1.0, r)
    perm = lambda t, l: g.view_4d(t, [d, l, h, b], [4, h * d * 4, d * 4, l * h * d * 4], 0)
    out = g.flash_attn_ext(perm(qd, lq), perm(kd, lk), perm(vd, lk), 1 / math.sqrt(d))
    try:
        nodes = g.build(out)
        assert gg.run(lib, nodes) == [0, 0, 0, 1]
        q = qd.numpy().reshape(b, lq, h * d)
        k = kd.numpy().reshape(b, lk, h * d)
        v = vd.numpy().reshape(b, lk, h * d)
        ex, mag = oracle.attention_exact(q, k, v, h, h, np.float32(1 / math.sqrt(d)))
        assert oracle.metric(out.numpy().reshape(ex.shape), ex, mag) <= oracle.K_B200
    finally:
        g.release(lib)


def test_other_threads_return_the_count_and_compute_nothing(lib):
    g = gg.Graph("host")
    r = oracle.generator(oracle.SEED)
    w = g.new_f16([64, 80], 0.25, r)
    x = g.new_f32([64, 40], 1.0, r)
    b = g.new_f32([80], 1.0, r)
    out = g.add_inplace(g.mul_mat(w, x), b)
    try:
        nodes = g.build(out)
        g.fill(nodes[0], np.full((1, 1, 40, 80), np.nan, dtype=np.float32))
        assert gg.compute_nodes(lib, nodes, 0, ith=1, nth=4) == 2
        assert np.isnan(out.numpy()).all()
        assert gg.compute_nodes(lib, nodes, 0, ith=0, nth=4) == 2
        ex, mag = oracle.mul_mat_exact(w.numpy()[0, 0], x.numpy()[0])
        bias = b.numpy().reshape(-1)
        assert oracle.metric(out.numpy()[0], ex + bias, mag + np.abs(bias)) <= oracle.K_B200
    finally:
        g.release(lib)


def test_compute_forward_single_node(lib):
    import ctypes

    g = gg.Graph("host")
    r = oracle.generator(oracle.SEED)
    x = g.new_f32([320, 64, 2], 3.0, r)
    y = g.norm(x, 1e-5)
    params = gg.ComputeParams(0, 1, 0, None, None, False)
    lib.sdasm_compute_forward.restype = ctypes.c_bool
    try:
        assert lib.sdasm_compute_forward(ctypes.byref(params), ctypes.byref(y.s))
        want = oracle.norm_ref(x.numpy(), 1e-5)
        assert np.abs(y.numpy() - want).max() <= 1e-6 * np.abs(want).max()
    finally:
        g.release(lib)


STORE_CASES = {
    "conv2d": lambda g, w: g.conv_2d_direct(w, g.new_f32([20, 12, 16, 2], 1.0, oracle.generator(100)),
                                            1, 1, 1, 1, 1, 1),
    "conv2d by Winograd": lambda g, w: g.conv_2d_direct(w, g.new_f32([64, 32, 16, 1], 1.0, oracle.generator(100)),
                                                        1, 1, 1, 1, 1, 1),
    "linear": lambda g, w: g.mul_mat(w, g.new_f32([64, 2000], 1.0, oracle.generator(100))),
}
STORE_WEIGHTS = {"conv2d": [3, 3, 16, 24], "conv2d by Winograd": [3, 3, 16, 24], "linear": [64, 80]}


@pytest.mark.parametrize("device", ["host", "cuda"])
@pytest.mark.parametrize("name", list(STORE_CASES))
def test_forget_makes_new_weights_used(lib, name, device):
    """ops_test.cc:643-719: weights set anew (and forgotten, as ggml's buffer write does)
    are used; a fresh computation with them agrees; without sdasm_forget the kept device
    copy of the old weights is what the kernels read."""
    def weights(g, seed):
        w = g.new_f16(STORE_WEIGHTS[name])
        g.fill(w, oracle.uniform(oracle.generator(seed), tuple(reversed(w.ne)), 1.0, np.float16))
        return w

    def reset(g, w, seed):
        g.fill(w, oracle.uniform(oracle.generator(seed), tuple(reversed(w.ne)), 1.0, np.float16))

    g = gg.Graph(device)
    g2 = gg.Graph(device)
    try:
        w = weights(g, 1)
        out = STORE_CASES[name](g, w)
        nodes = g.build(out)
        gg.run(lib, nodes)
        old = out.numpy()
        reset(g, w, 2)
        gg.forget(lib, w)
        gg.run(lib, nodes)
        changed = out.numpy()
        reset(g, w, 3)                  # no forget: the kept copy (and its packing) stays in use
        gg.run(lib, nodes)
        stale = out.numpy()
        out2 = STORE_CASES[name](g2, weights(g2, 2))
        gg.run(lib, g2.build(out2))
        fresh = out2.numpy()
    finally:
        g.release(lib)
        g2.release(lib)
    largest = np.abs(fresh).max()
    assert np.abs(changed - fresh).max() <= 1e-6 * largest
    assert np.abs(changed - old).max() > 1e-3 * largest
    assert np.array_equal(stale, changed)
