"""A float64 PyTorch restatement of the VAE decoder in stable-diffusion.assembly_b200/vae.py -- test infrastructure.

Same weights (read from the VAEDecoder object), standard NCHW formulas:
F.conv2d, F.group_norm (eps 1e-6), SiLU, single-head softmax attention over
the image's positions, nearest 2x upsampling.  The runner's result is compared
with this one.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

D = torch.float64


def _w(t):
    return t.to(D)


def gn(x, g, groups, eps, silu):
    y = F.group_norm(x, groups, _w(g[0]), _w(g[1]), eps)
    return F.silu(y) if silu else y


def resblock(x, rb, groups, eps):
    h = F.conv2d(gn(x, rb.gn1, groups, eps, True), _w(rb.conv1), _w(rb.b1), padding=1)
    h = F.conv2d(gn(h, rb.gn2, groups, eps, True), _w(rb.conv2), _w(rb.b2), padding=1)
    skip = x if rb.skip is None else F.conv2d(x, _w(rb.skip), _w(rb.bskip))
    return skip + h


def attention(x, at, groups, eps):
    b, c, h, w = x.shape
    n = gn(x, at.gn, groups, eps, False)
    q = F.conv2d(n, _w(at.wq), _w(at.bq)).reshape(b, c, h * w).transpose(1, 2)
    k = F.conv2d(n, _w(at.wk), _w(at.bk)).reshape(b, c, h * w).transpose(1, 2)
    v = F.conv2d(n, _w(at.wv), _w(at.bv)).reshape(b, c, h * w).transpose(1, 2)
    p = torch.softmax(q @ k.transpose(1, 2) / math.sqrt(c), dim=-1)
    o = (p @ v).transpose(1, 2).reshape(b, c, h, w)
    return x + F.conv2d(o, _w(at.wo), _w(at.bo))


def decode(vae, z):
    """z (N, h, w, 4) channels-last -> (N, 8h, 8w, 3) channels-last, float64."""
    c = vae.cfg
    x = z.to(D).permute(0, 3, 1, 2) / c.scale_factor
    x = F.conv2d(x, _w(vae.post_quant[0]), _w(vae.post_quant[1]))
    x = F.conv2d(x, _w(vae.conv_in[0]), _w(vae.conv_in[1]), padding=1)
    rb1, at, rb2 = vae.mid
    x = resblock(x, rb1, c.groups, c.eps)
    x = attention(x, at, c.groups, c.eps)
    x = resblock(x, rb2, c.groups, c.eps)
    for blocks, upsample in vae.up:
        for rb in blocks:
            x = resblock(x, rb, c.groups, c.eps)
        if upsample is not None:
            x = F.interpolate(x, scale_factor=2, mode="nearest")
            x = F.conv2d(x, _w(upsample[0]), _w(upsample[1]), padding=1)
    x = gn(x, vae.norm_out, c.groups, c.eps, True)
    x = F.conv2d(x, _w(vae.conv_out[0]), _w(vae.conv_out[1]), padding=1)
    return x.permute(0, 2, 3, 1)
