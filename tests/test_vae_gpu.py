"""The VAE decoder runner and the operations it adds: SOFT_MAX, products of two
operands the graph writes (sdb_mul_mat_transient), channel-major 1x1 outputs.

soft_max and the transient products are checked against float64 on their own;
the decoder -- a reduced configuration of SD 1.x's first-stage decoder --
against a float64 PyTorch restatement with the same weights
(tests/vae_reference.py) within 1e-5 of the largest output, as the UNet runner
is; the SD 1.5 decoder's attention block at full size (4096 positions, one
512-dim head) against float64; the full SD 1.5 decode (64 x 64 latent to
512 x 512) once eagerly and once from a CUDA graph, bit-identical.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

import oracle
from helpers import cuda_tensor, host, rng

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,cols,scale", [(64, 77, 0.125), (33, 1000, 1.0), (256, 4096, 1 / math.sqrt(512)),
                                             (7, 5000, 0.3), (3, 1, 1.0)])
def test_soft_max(cuda, rows, cols, scale):
    """Each row's softmax(scale x) within 4e-6 of float64, relative, where the exact weight is
    above 1e-30 (exponentials of FP32 arguments: the argument's own rounding, |scale x| 2^-24,
    and the exponential's last bits)."""
    import sdb

    g = rng(31)
    x = (g.standard_normal((rows, cols)) * 4).astype(np.float32)
    y = host(sdb.soft_max(cuda_tensor(x, cuda), scale))
    z = x.astype(np.float64) * np.float64(np.float32(scale))
    e = np.exp(z - z.max(axis=1, keepdims=True))
    e /= e.sum(axis=1, keepdims=True)
    big = e > 1e-30
    assert np.all(np.abs(y[big] - e[big]) <= 4e-6 * e[big])
    assert np.all(np.abs(y[~big]) <= 1e-30)


def test_soft_max_in_place_strided(cuda):
    """In place on a view whose rows are not contiguous with each other."""
    import sdb
    import torch

    g = torch.Generator(device=cuda).manual_seed(3)
    base = torch.randn(10, 300, device=cuda, generator=g)
    view = base[:, 50:250]
    want = torch.softmax(view.double() * 0.5, dim=-1)
    sdb.soft_max(view, 0.5, out=view)
    assert (view.double() - want).abs().max().item() <= 4e-6 * want.abs().max().item()
    assert bool(torch.isfinite(base).all())


@pytest.mark.parametrize("wtype", [np.float32, np.float16])
def test_mul_mat_transient_changes_between_calls(cuda, wtype):
    """The product against the exact oracle (<= 1e-6), and again after the first operand is
    overwritten in place: no packed copy of it is kept."""
    import sdb

    g = rng(32)
    w = oracle.uniform(g, (96, 300), 0.25, wtype)
    x = oracle.uniform(g, (2, 130, 300), 1.0)
    wt, xt = cuda_tensor(w, cuda), cuda_tensor(x, cuda)
    y1 = host(sdb.mul_mat_transient(wt, xt))
    ex, mag = oracle.mul_mat_exact(w, x)
    assert oracle.metric(y1, ex, mag) <= oracle.K_B200
    w2 = oracle.uniform(g, (96, 300), 0.25, wtype)
    wt.copy_(cuda_tensor(w2, cuda))
    y2 = host(sdb.mul_mat_transient(wt, xt))
    ex2, mag2 = oracle.mul_mat_exact(w2, x)
    assert oracle.metric(y2, ex2, mag2) <= oracle.K_B200
    e0, _ = sdb.store_stats()
    sdb.mul_mat_transient(wt, xt)
    assert sdb.store_stats()[0] == e0


def test_conv1x1_channel_major_output(cuda):
    """A 1x1 convolution of a channels-last image written channel-major (v^T of the VAE's attention)."""
    import sdb
    import torch

    g = rng(33)
    w = oracle.uniform(g, (48, 64, 1, 1), 0.25, np.float16)
    x = oracle.uniform(g, (2, 64, 12, 10), 1.0)
    b = oracle.uniform(g, (48,), 1.0)
    xt = cuda_tensor(x, cuda).permute(0, 2, 3, 1).contiguous()
    y = sdb.conv2d_nhwc(cuda_tensor(w, cuda), xt, out_nchw=True,
                        chain=sdb.Chain().add(cuda_tensor(b, cuda), [0, 0, 1, 0]))
    assert tuple(y.shape) == (2, 48, 12, 10)
    ex, mag = oracle.conv2d_exact(w, x)
    assert oracle.metric(host(y), ex + b.reshape(1, 48, 1, 1), mag + np.abs(b).reshape(1, 48, 1, 1)) <= oracle.K_B200


def test_vae_reduced_against_float64(cuda):
    import torch
    import vae as vae_mod
    import vae_reference

    cfg = vae_mod.VAEConfig(ch=32, ch_mult=(1, 2, 2), num_res_blocks=1)
    dec = vae_mod.VAEDecoder(cfg, device=cuda, seed=5)
    g = torch.Generator(device=cuda).manual_seed(6)
    z = torch.randn(2, 8, 8, 4, device=cuda, generator=g)
    got = dec.decode(z)
    want = vae_reference.decode(dec, z)
    assert tuple(got.shape) == (2, 32, 32, 3)
    err = (got.double() - want).abs().max().item()
    assert err <= 1e-5 * want.abs().max().item(), err


def test_sd15_vae_attention_full_size(cuda):
    """The SD 1.5 decoder's attention block (64 x 64 positions, one 512-dim head) against float64."""
    import torch
    import vae as vae_mod
    import vae_reference

    dec = vae_mod.VAEDecoder(device=cuda)
    at = dec.mid[1]
    g = torch.Generator(device=cuda).manual_seed(7)
    x = torch.randn(1, 64, 64, 512, device=cuda, generator=g)
    want = vae_reference.attention(x.double().permute(0, 3, 1, 2), at, 32, 1e-6).permute(0, 2, 3, 1)
    got = dec._attention(x.clone(), at)
    err = (got.double() - want).abs().max().item()
    assert err <= 1e-5 * want.abs().max().item(), err


def test_sd15_vae_decode_graph(cuda):
    """The full SD 1.5 decode, 64 x 64 latent to a 512 x 512 image: finite, and its CUDA-graph
    replay bit-identical to the eager decode."""
    import sdb
    import torch
    import vae as vae_mod

    dec = vae_mod.VAEDecoder(device=cuda)
    g = torch.Generator(device=cuda).manual_seed(8)
    z = torch.randn(1, 64, 64, 4, device=cuda, generator=g)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        eager = dec.decode(z).clone()
        dec.decode(z)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        out = dec.decode(z)
    graph.replay()
    torch.cuda.synchronize()
    assert tuple(eager.shape) == (1, 512, 512, 3)
    assert bool(torch.isfinite(eager).all())
    assert torch.equal(out, eager)
    assert sdb.device_status(clear=False) == 0


def test_sdxl_vae_attention_full_size(cuda):
    """The SDXL decoder's attention block at 832 x 1216 (152 x 104 positions, one 512-dim head) against
    float64."""
    import torch
    import vae as vae_mod
    import vae_reference

    dec = vae_mod.VAEDecoder(vae_mod.SDXL_VAE, device=cuda)
    at = dec.mid[1]
    g = torch.Generator(device=cuda).manual_seed(9)
    x = torch.randn(1, 152, 104, 512, device=cuda, generator=g)
    want = vae_reference.attention(x.double().permute(0, 3, 1, 2), at, 32, 1e-6).permute(0, 2, 3, 1)
    got = dec._attention(x.clone(), at)
    err = (got.double() - want).abs().max().item()
    assert err <= 1e-5 * want.abs().max().item(), err


def test_sdxl_vae_decode_full_size(cuda):
    """SDXL's decode, 152 x 104 latent to a 1216 x 832 image: finite, the latent's 1/0.13025 applied."""
    import torch
    import vae as vae_mod

    dec = vae_mod.VAEDecoder(vae_mod.SDXL_VAE, device=cuda)
    assert abs(dec.inv_scale.item() - 1 / 0.13025) <= 1e-6 / 0.13025
    g = torch.Generator(device=cuda).manual_seed(10)
    z = torch.randn(1, 152, 104, 4, device=cuda, generator=g)
    img = dec.decode(z)
    torch.cuda.synchronize()
    assert tuple(img.shape) == (1, 1216, 832, 3)
    assert bool(torch.isfinite(img).all())
