"""GroupNorm and LayerNorm fused into the operation that reads their output (sdb_group_norm_stats,
sdb_conv2d_normed, sdb_mul_mat_normed; sdb_mul_mat_layer_normed), against the reference's separate nodes.

The reference computes GROUP_NORM as a node of its own (norm.cc:100-140) between a convolution and the
next.  The fused path computes the group statistics once and normalises the input as the next
convolution (Winograd's input transform, or the split of a direct convolution's image) or linear layer
(the split of its rows) reads it.  The normalised numbers are those sdb_group_norm writes, so the fused
results must equal the separate nodes' bit for bit; the separate nodes are held to the oracle by
tests/test_norm_gpu.py and the convolution tests.  Checked here besides:
  * the statistics against the reference's single-precision mean and 1/sqrt(var + eps) (norm.cc:121-129);
  * benchmark config 2's shapes (conv 3x3 + bias -> GroupNorm 32 + SiLU -> the next conv) on the fused
    path against the float64 exact result of the reference's sequence, within the convolution bound.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from helpers import rng

pytestmark = pytest.mark.gpu


def nhwc(a):
    """(N, C, H, W) numpy -> channels-last torch tensor (N, H, W, C) on the GPU."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(np.transpose(a, (0, 2, 3, 1)))).cuda()


def affine(c, g):
    import torch

    gamma = torch.from_numpy(oracle.uniform(g, (c,), 1.0) + np.float32(1.0)).cuda()
    beta = torch.from_numpy(oracle.uniform(g, (c,), 1.0)).cuda()
    return gamma, beta


def separate_gn(x, gamma, beta, groups, eps, silu):
    import sdb

    ch = sdb.Chain().mul(gamma, [0, 0, 1, 0]).add(beta, [0, 0, 1, 0])
    if silu:
        ch.silu()
    return sdb.group_norm_nhwc(x, groups, eps, chain=ch)


@pytest.mark.parametrize("shape,groups,eps", [((2, 320, 64, 64), 32, 1e-5), ((3, 640, 17, 9), 32, 1e-6),
                                              ((1, 1280, 8, 8), 32, 1e-5), ((2, 96, 5, 7), 8, 1e-5)])
def test_group_norm_stats_are_the_reference_statistics(cuda, shape, groups, eps):
    import sdb

    g = rng(11)
    x = oracle.uniform(g, shape, 3.0) + np.float32(1.5)
    st = sdb.group_norm_stats(nhwc(x), groups, eps).cpu().numpy()
    n, c = shape[:2]
    per = c // groups
    for i in range(n):
        for k in range(groups):
            grp = x[i, k * per:(k + 1) * per].reshape(-1)
            mean = np.float32(grp.astype(np.float64).sum() / grp.size)
            d = (grp - mean).astype(np.float32)
            var = np.float32((d * d).astype(np.float64).sum() / grp.size)
            scale = np.float32(1.0) / np.sqrt(np.float32(var + np.float32(eps)), dtype=np.float32)
            assert abs(st[i, k, 0] - mean) <= 2e-7 * max(1.0, abs(mean)), (i, k)
            assert abs(st[i, k, 1] - scale) <= 1e-6 * scale, (i, k)


# (n, ic, oc, h, w, kernel, padding): Winograd F(4x4) (64x64, 32x32), F(2x2)-free 16x16 direct, 8x8 direct,
# a 1x1 convolution, an odd image.
CONVS = [(2, 320, 320, 64, 64, 3, 1), (2, 640, 640, 32, 32, 3, 1), (2, 1280, 1280, 16, 16, 3, 1),
         (1, 1280, 1280, 8, 8, 3, 1), (2, 640, 320, 32, 32, 1, 0), (1, 96, 64, 13, 11, 3, 1)]


@pytest.mark.parametrize("case", CONVS, ids=lambda c: "x".join(map(str, c)))
def test_conv_normed_equals_separate_nodes(cuda, case):
    """conv(SiLU(GroupNorm(x))) fused is the separate nodes' result bit for bit."""
    import sdb
    import torch

    n, ic, oc, h, w, k, p = case
    g = rng(12)
    x = nhwc(oracle.uniform(g, (n, ic, h, w), 2.0) + np.float32(0.5))
    wt = torch.from_numpy(oracle.uniform(g, (oc, ic, k, k), 1.0 / (3 * np.sqrt(ic)), np.float16)).cuda()
    b = torch.from_numpy(oracle.uniform(g, (oc,), 0.1)).cuda()
    gamma, beta = affine(ic, g)
    chain = sdb.Chain().add(b, [0, 0, 1, 0])
    fused = sdb.conv2d_nhwc_normed(wt, x, sdb.GroupNormIn(sdb.group_norm_stats(x, 32, 1e-5), 32, gamma, beta, True),
                                   (1, 1), (p, p), chain=chain)
    apart = sdb.conv2d_nhwc(wt, separate_gn(x, gamma, beta, 32, 1e-5, True), (1, 1), (p, p), chain=chain)
    torch.cuda.synchronize()
    assert torch.isfinite(fused).all()
    assert torch.equal(fused, apart)


@pytest.mark.parametrize("n,c,hw,silu", [(2, 640, 32 * 32, False), (1, 320, 77, True), (3, 1280, 64, False)])
def test_mul_mat_normed_equals_separate_nodes(cuda, n, c, hw, silu):
    """The transformer's proj_in of GroupNorm(x) (eps 1e-6, no SiLU) fused is the separate nodes' result."""
    import sdb
    import torch

    g = rng(13)
    x = torch.from_numpy(oracle.uniform(g, (n, hw, c), 2.0)).cuda()          # (N, P, C): channels-last rows
    w = torch.from_numpy(oracle.uniform(g, (c, c), 0.25 / np.sqrt(c), np.float16)).cuda()
    b = torch.from_numpy(oracle.uniform(g, (c,), 0.1)).cuda()
    gamma, beta = affine(c, g)
    img = x.view(n, hw, 1, c)                                                 # (N, H=P, W=1, C)
    stats = sdb.group_norm_stats(img, 32, 1e-6)
    fused = sdb.mul_mat_normed(w, x, sdb.GroupNormIn(stats, 32, gamma, beta, silu), chain=sdb.Chain().add(b))
    normed = separate_gn(img, gamma, beta, 32, 1e-6, silu).view(n, hw, c)
    apart = sdb.mul_mat(w, normed, chain=sdb.Chain().add(b))
    torch.cuda.synchronize()
    assert torch.equal(fused, apart)


@pytest.mark.parametrize("c,hw", [(320, 64), (640, 32), (1280, 8)], ids=["2a", "2b", "2c"])
def test_config2_block_fused_within_bound(cuda, c, hw):
    """benchmark config 2 as the UNet runs it: conv 3x3 + bias, GroupNorm(32, eps 1e-5, gamma ~ N(1, 0.1),
    beta ~ N(0, 0.1)) + SiLU applied as the next convolution reads it.  The result against float64:
    the exact second convolution of the oracle's GroupNorm + SiLU of the first's exact output, bounded
    as the convolution tests bound a single convolution (plus the first's error carried through)."""
    import sdb
    import torch

    g = np.random.default_rng(2024)
    x = g.standard_normal((1, c, hw, hw)).astype(np.float32)
    w1 = (g.standard_normal((c, c, 3, 3)) / np.sqrt(9 * c)).astype(np.float16)
    w2 = (g.standard_normal((c, c, 3, 3)) / np.sqrt(9 * c)).astype(np.float16)
    b1 = (g.standard_normal(c) * 0.02).astype(np.float32)
    gamma = (1 + 0.1 * g.standard_normal(c)).astype(np.float32)
    beta = (0.1 * g.standard_normal(c)).astype(np.float32)
    tw1, tw2 = torch.from_numpy(w1).cuda(), torch.from_numpy(w2).cuda()
    tb1, tg, tbt = (torch.from_numpy(a).cuda() for a in (b1, gamma, beta))
    y = sdb.conv2d_nhwc(tw1, nhwc(x), (1, 1), (1, 1), chain=sdb.Chain().add(tb1, [0, 0, 1, 0]))
    z = sdb.conv2d_nhwc_normed(tw2, y, sdb.GroupNormIn(sdb.group_norm_stats(y, 32, 1e-5), 32, tg, tbt, True),
                               (1, 1), (1, 1))
    torch.cuda.synchronize()
    got = z.cpu().numpy().transpose(0, 3, 1, 2)
    # The reference's sequence in float64 from the first convolution's exact output.
    y_ex, _ = oracle.conv2d_exact(w1, x, (1, 1), (1, 1), (1, 1))
    y_ex = (y_ex + b1.reshape(1, -1, 1, 1)).astype(np.float64)
    t = oracle.group_norm_exact(y_ex, 32, 1e-5) * gamma.reshape(1, -1, 1, 1) + beta.reshape(1, -1, 1, 1)
    t = t / (1.0 + np.exp(-t))
    z_ex, z_mag = oracle.conv2d_exact(w2, t, (1, 1), (1, 1), (1, 1))
    err = oracle.metric(got, z_ex, z_mag)
    # The first convolution's own error (<= its bound, relative to its magnitudes) passes through the
    # normalisation (scale 1/std) and the second convolution: a few times 1e-6 of the magnitudes.
    assert err <= 5e-6, f"error {err:.3g}"


@pytest.mark.parametrize("rows,k,n,gated", [(2 * 4096, 320, 960, False), (77, 640, 640, False), (300, 1280, 2 * 1280, True),
                                            (33, 40, 24, False)])
def test_linear_layer_normed_equals_separate_nodes(cuda, rows, k, n, gated):
    """LayerNorm (eps 1e-5, gamma and beta) fused into the split of the next linear layer (or GEGLU) equals
    sdb_norm followed by the layer, bit for bit."""
    import sdb
    import torch

    g = rng(14)
    x = torch.from_numpy(oracle.uniform(g, (rows, k), 3.0) + np.float32(0.25)).cuda()
    w = torch.from_numpy(oracle.uniform(g, (n, k), 0.25 / np.sqrt(k), np.float16)).cuda()
    b = torch.from_numpy(oracle.uniform(g, (n,), 0.1)).cuda()
    gamma, beta = affine(k, g)
    ln = sdb.Chain().mul(gamma).add(beta)
    fused = sdb.mul_mat_layer_normed(w, x, 1e-5, ln, chain=sdb.Chain().add(b), gated=gated)
    h = sdb.norm(x, 1e-5, chain=ln)
    apart = (sdb.mul_mat_gated if gated else sdb.mul_mat)(w, h, chain=sdb.Chain().add(b))
    torch.cuda.synchronize()
    assert torch.isfinite(fused).all()
    assert torch.equal(fused, apart)
    # And the separate LayerNorm is the reference's (norm.cc:148-175) within 1e-6 of its largest output.
    want = oracle.apply_chain(oracle.norm_ref(x.cpu().numpy()[:64], 1e-5),
                              [("mul", gamma.cpu().numpy()), ("add", beta.cpu().numpy())])
    assert np.abs(h.cpu().numpy()[:64] - want).max() <= 1e-6 * np.abs(want).max()
