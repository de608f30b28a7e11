"""A float64 PyTorch restatement of the UNet in stable-diffusion.assembly_b200/unet.py -- test infrastructure.

Same weights (read from the UNet object), standard NCHW formulas: F.conv2d,
F.group_norm, F.layer_norm, softmax attention per head, GELU in its tanh form
(the reference's scalar_math.h gelu), SiLU, nearest upsampling, the timestep
embedding as [cos | sin].  The runner's result is compared with this one.
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


def resblock(x, rb, emb, groups):
    h = F.conv2d(gn(x, rb.gn1, groups, 1e-5, True), _w(rb.conv1), _w(rb.b1), padding=1)
    h = h + emb[:, rb.emb_offset:rb.emb_offset + rb.cout, None, None]
    h = F.conv2d(gn(h, rb.gn2, groups, 1e-5, True), _w(rb.conv2), _w(rb.b2), padding=1)
    skip = x if rb.skip is None else F.conv2d(x, _w(rb.skip), _w(rb.bskip))
    return skip + h


def attention(q, k, v, heads):
    b, lq, c = q.shape
    d = c // heads
    q = q.view(b, lq, heads, d).transpose(1, 2)
    k = k.view(b, k.shape[1], heads, d).transpose(1, 2)
    v = v.view(b, v.shape[1], heads, d).transpose(1, 2)
    p = torch.softmax((q @ k.transpose(-1, -2)) / math.sqrt(d), dim=-1)
    return (p @ v).transpose(1, 2).reshape(b, lq, c)


def transformer(x, tr, context, groups, todo=(1, 4096)):
    """todo (factor, least tokens): ToDo's keys and values from every factor-th token of every
    factor-th row of grids of at least that many tokens (stable-diffusion.cpp patch 0004)."""
    b, c, h, w = x.shape
    heads = tr.heads
    f = todo[0] if todo[0] >= 2 and h * w >= todo[1] else 1
    n = gn(x, tr.gn, groups, 1e-6, False)
    t = n.permute(0, 2, 3, 1).reshape(b, h * w, c) @ _w(tr.proj_in).T + _w(tr.b_in)
    for blk in tr.blocks:
        h1 = F.layer_norm(t, (c,), _w(blk.ln1[0]), _w(blk.ln1[1]), 1e-5)
        wqkv = _w(blk.wqkv).T
        src = h1.view(b, h, w, c)[:, ::f, ::f, :].reshape(b, -1, c) if f > 1 else h1
        kv = src @ wqkv[:, c:]
        a = attention(h1 @ wqkv[:, :c], kv[..., :c], kv[..., c:], heads)
        t = t + a @ _w(blk.wo1).T + _w(blk.bo1)
        h2 = F.layer_norm(t, (c,), _w(blk.ln2[0]), _w(blk.ln2[1]), 1e-5)
        kv = context @ _w(blk.kv_w).T
        t = t + attention(h2 @ _w(blk.wq2).T, kv[..., :c], kv[..., c:], heads) @ _w(blk.wo2).T + _w(blk.bo2)
        h3 = F.layer_norm(t, (c,), _w(blk.ln3[0]), _w(blk.ln3[1]), 1e-5)
        y = h3 @ _w(blk.wff1).T + _w(blk.bff1)
        g = y[..., :4 * c] * F.gelu(y[..., 4 * c:], approximate="tanh")
        t = t + g @ _w(blk.wff2).T + _w(blk.bff2)
    out = t @ _w(tr.proj_out).T + _w(tr.b_out)
    return x + out.view(b, h, w, c).permute(0, 3, 1, 2)


def timestep_embedding(t, dim, max_period=10000):
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=D, device=t.device) / half)
    args = t.to(D)[:, None] * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


def forward(unet, x_nhwc, timesteps, context, y=None, todo=(1, 4096)):
    """eps (B, H, W, C_out) in float64 for the runner's weights and inputs (y: the label embedding's input;
    todo: ToDo's factor and least tokens, as the tuning's todo and todo_tokens)."""
    cfg = unet.cfg
    groups = cfg.groups
    # The fused K/V weights, split back per block.
    for tr in unet.transformers:
        for blk in tr.blocks:
            blk.kv_w = unet.kv_w[blk.kv_offset:blk.kv_offset + 2 * tr.c]
    te = timestep_embedding(timesteps, cfg.model_channels)
    e = F.silu(te @ _w(unet.t_w1).T + _w(unet.t_b1))
    e = e @ _w(unet.t_w2).T + _w(unet.t_b2)
    if cfg.adm_in_channels:
        lab = F.silu(y.to(D) @ _w(unet.label_w1).T + _w(unet.label_b1))
        e = e + lab @ _w(unet.label_w2).T + _w(unet.label_b2)
    e = F.silu(e)
    emb = e @ _w(unet.emb_w).T + _w(unet.emb_b)
    ctx = context.to(D)
    h = F.conv2d(x_nhwc.to(D).permute(0, 3, 1, 2), _w(unet.conv_in), _w(unet.conv_in_b), padding=1)
    hs = [h]
    for level in unet.down:
        for rb, tr in level.blocks:
            h = resblock(h, rb, emb, groups)
            if tr is not None:
                h = transformer(h, tr, ctx, groups, todo)
            hs.append(h)
        if level.down is not None:
            h = F.conv2d(h, _w(level.down[0]), _w(level.down[1]), stride=2, padding=1)
            hs.append(h)
    rb1, tr, rb2 = unet.mid
    h = resblock(h, rb1, emb, groups)
    h = transformer(h, tr, ctx, groups, todo)
    h = resblock(h, rb2, emb, groups)
    for level in unet.up:
        for rb, tr in level.blocks:
            h = torch.cat([h, hs.pop()], dim=1)
            h = resblock(h, rb, emb, groups)
            if tr is not None:
                h = transformer(h, tr, ctx, groups, todo)
        if level.up is not None:
            h = F.interpolate(h, scale_factor=2, mode="nearest")
            h = F.conv2d(h, _w(level.up[0]), _w(level.up[1]), padding=1)
    h = F.conv2d(gn(h, unet.out_gn, groups, 1e-5, True), _w(unet.conv_out), _w(unet.conv_out_b), padding=1)
    return h.permute(0, 2, 3, 1)
