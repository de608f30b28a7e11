"""The device-resident UNet runner and its glue kernels.

The glue nodes (concat, nearest upscale, timestep embedding, guidance + Euler
update) are checked exactly against their definitions; the whole UNet -- a
reduced configuration of the SD 1.x architecture -- against a float64 PyTorch
restatement of the same network with the same weights (tests/unet_reference.py),
within 1e-5 of the largest output: each of its ~60 operations is held to the
1e-6 metric on its own (the other test files), and errors of that size compound
through the residual stream.  The full SD 1.5 UNet runs once at its benchmark
shape (batch 2, 64 x 64 latent) and its graph replay is compared with the eager
forward.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_concat_upscale_timestep(cuda):
    import sdb
    import torch

    g = torch.Generator(device=cuda).manual_seed(1)
    a = torch.randn(2, 8, 8, 96, device=cuda, generator=g)
    b = torch.randn(2, 8, 8, 32, device=cuda, generator=g)
    assert torch.equal(sdb.concat_channels_nhwc(a, b), torch.cat([a, b], dim=3))
    odd = torch.randn(2, 5, 3, 7, device=cuda, generator=g)
    odd2 = torch.randn(2, 5, 3, 6, device=cuda, generator=g)
    assert torch.equal(sdb.concat_channels_nhwc(odd, odd2), torch.cat([odd, odd2], dim=3))
    up = sdb.upscale_nearest_nhwc(a, 2)
    assert torch.equal(up, a.repeat_interleave(2, dim=1).repeat_interleave(2, dim=2))
    t = torch.tensor([0.0, 1.5, 999.0], device=cuda)
    emb = sdb.timestep_embedding(t, 320)
    half = 160
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float64, device=cuda) / half)
    args = t.double()[:, None] * freqs[None]
    want = torch.cat([torch.cos(args), torch.sin(args)], dim=1)
    # Float arguments of up to 999 rad: the phase itself carries ~1e-4 of rounding.
    assert (emb.double() - want).abs().max().item() < 2e-4


def test_euler_cfg_step(cuda):
    import sdb
    import torch

    g = torch.Generator(device=cuda).manual_seed(2)
    n = 4 * 64 * 64
    eps = torch.randn(2, n, device=cuda, generator=g)
    x = torch.randn(n, device=cuda, generator=g)
    x_in = torch.empty(2, n, device=cuda)
    x0 = x.clone()
    sdb.euler_cfg_step(eps, x, x_in, 7.0, 14.6, 11.2, 0.25)
    e = eps[0] + 7.0 * (eps[1] - eps[0])
    want = x0 + (11.2 - 14.6) * e
    torch.testing.assert_close(x, want, rtol=1e-6, atol=1e-5)
    torch.testing.assert_close(x_in[0], want * 0.25, rtol=1e-6, atol=1e-5)
    torch.testing.assert_close(x_in[1], want * 0.25, rtol=1e-6, atol=1e-5)


@pytest.mark.parametrize("sigma,sigma_next", [(14.6, 11.2), (0.9, 0.0)])
def test_euler_ancestral_cfg_step(cuda, sigma, sigma_next):
    """The ancestral step (k-diffusion's sample_euler_ancestral, eta 1) against its formula in double:
    sigma_up, sigma_down, the deterministic part to sigma_down and the fresh noise times sigma_up (none
    at the last step)."""
    import sdb
    import torch

    g = torch.Generator(device=cuda).manual_seed(4)
    n = 4 * 152 * 104
    eps = torch.randn(2, n, device=cuda, generator=g)
    x = torch.randn(n, device=cuda, generator=g)
    noise = torch.randn(n, device=cuda, generator=g)
    x_in = torch.empty(2, n, device=cuda)
    x0 = x.clone()
    sdb.euler_ancestral_cfg_step(eps, x, x_in, noise, 6.0, sigma, sigma_next, 0.5)
    up = min(sigma_next, math.sqrt(sigma_next ** 2 * (sigma ** 2 - sigma_next ** 2) / sigma ** 2))
    down = math.sqrt(sigma_next ** 2 - up ** 2)
    e = eps[0].double() + 6.0 * (eps[1].double() - eps[0].double())
    want = x0.double() + (down - sigma) * e + up * noise.double()
    assert (x.double() - want).abs().max().item() <= 1e-5 * max(1.0, want.abs().max().item())
    torch.testing.assert_close(x_in[0], x * 0.5, rtol=0, atol=0)
    torch.testing.assert_close(x_in[1], x * 0.5, rtol=0, atol=0)


TINY = dict(model_channels=32, channel_mult=(1, 2), num_res_blocks=1, attention_levels=(1,), heads=2,
            context_dim=32, groups=8)


def test_unet_tiny_matches_float64(cuda):
    import torch
    import unet as U
    import unet_reference as R

    net = U.UNet(U.UNetConfig(**TINY), device=cuda, seed=5)
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(2, 16, 16, 4, device=cuda, generator=g)
    t = torch.tensor([981.0, 981.0], device=cuda)
    ctx = torch.randn(2, 8, 32, device=cuda, generator=g)
    got = net.forward(x, t, ctx).double()
    torch.cuda.synchronize()
    want = R.forward(net, x, t, ctx)
    err = (got - want).abs().max().item() / want.abs().max().item()
    assert np.isfinite(err) and err <= 1e-5, f"{err:.3g} of the largest output"


# The SDXL structure made small: no attention at the first level, transformers of depth 2 (and 2 in the
# middle) with heads of a fixed width, the label embedding added to the time embedding.
TINY_XL = dict(model_channels=32, channel_mult=(1, 2), num_res_blocks=1, attention_levels=(1,),
               transformer_depth=(0, 2), mid_depth=2, head_dim=16, context_dim=48, groups=8, adm_in_channels=40)


def test_unet_tiny_sdxl_structure_matches_float64(cuda):
    import torch
    import unet as U
    import unet_reference as R

    net = U.UNet(U.UNetConfig(**TINY_XL), device=cuda, seed=6)
    g = torch.Generator(device=cuda).manual_seed(9)
    x = torch.randn(2, 16, 16, 4, device=cuda, generator=g)
    t = torch.tensor([500.0, 500.0], device=cuda)
    ctx = torch.randn(2, 9, 48, device=cuda, generator=g)
    y = torch.randn(2, 40, device=cuda, generator=g)
    got = net.forward(x, t, ctx, y=y).double()
    torch.cuda.synchronize()
    want = R.forward(net, x, t, ctx, y=y)
    err = (got - want).abs().max().item() / want.abs().max().item()
    assert np.isfinite(err) and err <= 1e-5, f"{err:.3g} of the largest output"


def test_sdxl_unet_forward(cuda):
    """The SDXL UNet (2.57B parameters) once at a 64 x 64 latent, batch 2: finite, graph replay bit-identical."""
    import torch
    import unet as U

    net = U.UNet(U.SDXL, device=cuda, seed=8)
    assert 2.5e9 < net.params < 2.65e9, net.params
    g = torch.Generator(device=cuda).manual_seed(10)
    x = torch.randn(2, 64, 64, 4, device=cuda, generator=g)
    t = torch.tensor([700.0, 700.0], device=cuda)
    ctx = torch.randn(2, 77, 2048, device=cuda, generator=g)
    y = torch.randn(2, 2816, device=cuda, generator=g)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        eager = net.forward(x, t, ctx, y=y).clone()
        net.forward(x, t, ctx, y=y)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        out = net.forward(x, t, ctx, y=y)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.isfinite(eager).all()
    assert torch.equal(out, eager)
    del graph


def test_sd15_unet_graph_replay(cuda):
    """SD 1.5 at its benchmark shape: the captured step equals the eager forward, bit for bit."""
    import torch
    import unet as U

    net = U.UNet(U.SD15, device=cuda, seed=7)
    assert 8.4e8 < net.params < 8.8e8, net.params   # ~860M parameters
    sampler = U.Sampler(net, 64, 64, steps=2)
    g = torch.Generator(device=cuda).manual_seed(4)
    sampler.x.copy_(torch.randn(1, 64, 64, 4, device=cuda, generator=g))
    sampler.context.copy_(torch.randn(2, 77, 768, device=cuda, generator=g))
    sampler.set_step(0)
    eager = sampler.step_forward().clone()
    sampler.capture()
    replay = sampler.step_forward().clone()
    torch.cuda.synchronize()
    assert torch.isfinite(eager).all()
    assert torch.equal(eager, replay)
    assert eager.abs().max().item() < 1e4


@pytest.mark.parametrize("factor", [2, 3])
def test_unet_tiny_todo_matches_float64(cuda, factor):
    """ToDo (todo=2 or 3): self-attention's keys and values from every f-th token of every f-th row
    of the transformers' 8 x 8 grids (todo_tokens lowered to 64); against the float64 restatement with
    the same rule."""
    import sdb
    import torch
    import unet as U
    import unet_reference as R

    net = U.UNet(U.UNetConfig(**TINY), device=cuda, seed=5)
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(2, 16, 16, 4, device=cuda, generator=g)
    t = torch.tensor([981.0, 981.0], device=cuda)
    ctx = torch.randn(2, 8, 32, device=cuda, generator=g)
    sdb.set_tuning(f"todo={factor},todo_tokens=64")
    try:
        assert sdb.token_downsampling(8, 8) == factor and sdb.token_downsampling(7, 9) == 1
        got = net.forward(x, t, ctx).double()
        torch.cuda.synchronize()
    finally:
        sdb.set_tuning("todo=1,todo_tokens=4096")
    want = R.forward(net, x, t, ctx, todo=(factor, 64))
    plain = R.forward(net, x, t, ctx)
    err = (got - want).abs().max().item() / want.abs().max().item()
    assert np.isfinite(err) and err <= 1e-5, f"{err:.3g} of the largest output"
    # And it is not the full attention.
    assert (plain - want).abs().max().item() > 1e3 * (got - want).abs().max().item()


def test_coarser_tokens(cuda):
    """sdb_coarser_tokens against slicing, a grid of odd size (ceil), channels of no multiple of 4."""
    import sdb
    import torch

    for c in (8, 6):
        x = torch.randn(2, 7 * 5, c, device=cuda)
        y = sdb.coarser_tokens(x, 5, 7, 2)
        want = x.view(2, 7, 5, c)[:, ::2, ::2, :].reshape(2, -1, c)
        assert torch.equal(y, want)


def test_sd15_unet_eight_images(cuda):
    """The bench's per-GPU batch at one GPU: SD 1.5's UNet on 8 images' guidance batch (16) gives each
    image's pair what the pair alone gives (within 1e-5 of the largest output: only the GEMMs' plans,
    split by the row count, differ)."""
    import torch
    import unet as U

    net = U.UNet(U.SD15, device=cuda, seed=20261011)
    g = torch.Generator(device=cuda).manual_seed(21)
    x = torch.randn(16, 64, 64, 4, device=cuda, generator=g)
    t = torch.full((16,), 500.0, device=cuda)
    ctx = torch.randn(16, 77, 768, device=cuda, generator=g)
    eps = net.forward(x, t, ctx)
    for i in (0, 5):
        rows = [i, 8 + i]
        pair = net.forward(x[rows].contiguous(), t[rows].contiguous(), ctx[rows].contiguous())
        err = (eps[rows] - pair).abs().max().item() / pair.abs().max().item()
        assert err <= 1e-5, f"image {i}: {err:.3g}"
    del net
    torch.cuda.empty_cache()


def test_sd15_unet_fused_norms_equal_separate_nodes(cuda):
    """SD 1.5's forward with its GroupNorms and LayerNorms fused into the convolution or linear layer
    that reads them (sdb_group_norm_stats + sdb_conv2d_normed / sdb_mul_mat_normed,
    sdb_mul_mat_layer_normed) equals the forward with the reference's separate GROUP_NORM and NORM
    nodes, bit for bit."""
    import torch
    import unet as U

    net = U.UNet(U.SD15, device=cuda, seed=7)
    g = torch.Generator(device=cuda).manual_seed(12)
    x = torch.randn(2, 64, 64, 4, device=cuda, generator=g)
    t = torch.tensor([600.0, 600.0], device=cuda)
    ctx = torch.randn(2, 77, 768, device=cuda, generator=g)
    net.fuse_gn = net.fuse_ln = True
    fused = net.forward(x, t, ctx).clone()
    net.fuse_gn = net.fuse_ln = False
    apart = net.forward(x, t, ctx).clone()
    net.fuse_gn = net.fuse_ln = True
    torch.cuda.synchronize()
    assert torch.isfinite(fused).all()
    assert torch.equal(fused, apart)
