"""The SD 1.x VAE decoder (AutoencoderKL's Decoder) on the library's kernels.

stable-diffusion.cpp decodes the sampled latent with the VAE's decoder graph:
3x3 convolutions (CONV_2D), GroupNorm with SiLU, nearest 2x upsampling, and one
self-attention block at the latent's resolution with a single 512-dim head.
sdb_attention takes heads of up to 160 dims, so that head runs in the form of
a graph without flash attention: MUL_MAT (k.q), SOFT_MAX, MUL_MAT (v.p) -- all
three nodes the reference leaves or hands to its own MUL_MAT.  Here the same
network runs device-resident, channels-last (N, H, W, C):

  * convolutions: sdb_conv2d (Winograd F(4x4) or direct, by the tuning), bias,
    residual and the 1/scale_factor of the latent in their chains;
  * GroupNorm (eps 1e-6, affine, SiLU): sdb_group_norm on channels-last images;
  * the attention block: q and k as 1x1 convolutions into token rows, v as a
    1x1 convolution written channel-major (v^T, the layout ggml's graph gives
    it), then k.q and v.softmax(k.q) by sdb_mul_mat_transient (operands the
    graph writes, never kept by the weight store) and sdb_soft_max, the output
    projection adding into the block's input;
  * upsampling: sdb_upscale_nearest.

The architecture is SD 1.x's first-stage decoder: z 4 channels, ch 128,
ch_mult 1/2/4/4, 2 ResBlocks a level (+1 in the decoder), attention in the
middle only, GroupNorm 32 (eps 1e-6), scale factor 0.18215.  A 64 x 64 latent
decodes to a 512 x 512 image.  Weights are random (the benchmark's random-init
FP16 weights), drawn from one seed on the device.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import sdb
from unet import _Init


@dataclass(frozen=True)
class VAEConfig:
    z_channels: int = 4
    out_channels: int = 3
    ch: int = 128
    ch_mult: tuple = (1, 2, 4, 4)
    num_res_blocks: int = 2
    groups: int = 32
    eps: float = 1e-6
    scale_factor: float = 0.18215


SD15_VAE = VAEConfig()
# SDXL's first-stage decoder: the same network, its latents scaled by 0.13025.
SDXL_VAE = VAEConfig(scale_factor=0.13025)


@dataclass
class VResBlock:
    cin: int
    cout: int
    gn1: tuple
    conv1: object
    b1: object
    gn2: tuple
    conv2: object
    b2: object
    skip: object = None
    bskip: object = None


@dataclass
class VAttn:
    c: int
    gn: tuple
    wq: object
    bq: object
    wk: object
    bk: object
    wv: object
    bv: object
    wo: object
    bo: object
    wo_lin: object = None     # wo as a (C, C) linear weight: one view object, so the store keeps one packing


class VAEDecoder:
    """decode(z (N, h, w, 4)) -> image (N, 8h, 8w, 3), channels-last, before the [-1, 1] -> [0, 1] clamp."""

    def __init__(self, config: VAEConfig = SD15_VAE, device="cuda", seed: int = 20261012):
        import torch

        self.torch = torch
        self.cfg = config
        self.device = torch.device(device)
        init = _Init(self.device, seed)
        c = config

        def resblock(cin, cout):
            rb = VResBlock(cin, cout, (init.gamma(cin), init.beta(cin)), init.conv(cout, cin, 3), init.bias(cout),
                           (init.gamma(cout), init.beta(cout)), init.conv(cout, cout, 3), init.bias(cout))
            if cin != cout:
                rb.skip, rb.bskip = init.conv(cout, cin, 1), init.bias(cout)
            return rb

        block_in = c.ch * c.ch_mult[-1]
        self.post_quant = (init.conv(c.z_channels, c.z_channels, 1), init.bias(c.z_channels))
        self.conv_in = (init.conv(block_in, c.z_channels, 3), init.bias(block_in))
        attn = VAttn(block_in, (init.gamma(block_in), init.beta(block_in)),
                     init.conv(block_in, block_in, 1), init.bias(block_in),
                     init.conv(block_in, block_in, 1), init.bias(block_in),
                     init.conv(block_in, block_in, 1), init.bias(block_in),
                     init.conv(block_in, block_in, 1), init.bias(block_in))
        attn.wo_lin = attn.wo.view(block_in, block_in)
        self.mid = (resblock(block_in, block_in), attn, resblock(block_in, block_in))
        self.up = []  # in decoding order: deepest level first
        for lvl in reversed(range(len(c.ch_mult))):
            block_out = c.ch * c.ch_mult[lvl]
            blocks = []
            for _ in range(c.num_res_blocks + 1):
                blocks.append(resblock(block_in, block_out))
                block_in = block_out
            upsample = (init.conv(block_in, block_in, 3), init.bias(block_in)) if lvl != 0 else None
            self.up.append((blocks, upsample))
        self.norm_out = (init.gamma(block_in), init.beta(block_in))
        self.conv_out = (init.conv(c.out_channels, block_in, 3), init.bias(c.out_channels))
        self.inv_scale = torch.full((1,), 1.0 / c.scale_factor, device=self.device, dtype=torch.float32)
        self.params = init.params

    # ------------------------------------------------------------ pieces

    def _gn(self, x, gn, silu, out=None):
        ch = sdb.Chain().mul(gn[0], [0, 0, 1, 0]).add(gn[1], [0, 0, 1, 0])
        if silu:
            ch.silu()
        return sdb.group_norm_nhwc(x, self.cfg.groups, self.cfg.eps, out=out, chain=ch)

    def _conv3(self, w, b, x, out=None, chain=None):
        ch = sdb.Chain().add(b, [0, 0, 1, 0]) if chain is None else chain
        return sdb.conv2d_nhwc(w, x, (1, 1), (1, 1), out=out, chain=ch)

    def _resblock(self, x, rb: VResBlock):
        t1 = self._gn(x, rb.gn1, True)
        h = self._conv3(rb.conv1, rb.b1, t1)
        t2 = self._gn(h, rb.gn2, True, out=t1 if rb.cin == rb.cout else None)
        if rb.skip is None:
            xs = (x.stride(2), x.stride(1), x.stride(3), x.stride(0))  # ggml order [W, H, C, N]
            return self._conv3(rb.conv2, None, t2, out=h, chain=sdb.Chain().add(rb.b2, [0, 0, 1, 0]).add(x, list(xs)))
        out = sdb.conv2d_nhwc(rb.skip, x, chain=sdb.Chain().add(rb.bskip, [0, 0, 1, 0]))
        self._conv3(rb.conv2, None, t2, out=h, chain=sdb.Chain().add(rb.b2, [0, 0, 1, 0]).redirect(out, True))
        return out

    def _attention(self, x, at: VAttn):
        """x + proj_out(softmax(q k^T / sqrt(C)) v), one head of C dims over the image's positions."""
        b, hh, ww, c = x.shape
        n = self._gn(x, at.gn, False)
        lq = hh * ww
        q = sdb.conv2d_nhwc(at.wq, n, chain=sdb.Chain().add(at.bq, [0, 0, 1, 0]))
        k = sdb.conv2d_nhwc(at.wk, n, chain=sdb.Chain().add(at.bk, [0, 0, 1, 0]))
        vt = sdb.conv2d_nhwc(at.wv, n, out_nchw=True, chain=sdb.Chain().add(at.bv, [0, 0, 1, 0]))
        for i in range(b):
            s = sdb.mul_mat_transient(k[i].view(lq, c), q[i].view(lq, c))      # s[i][j] = q_i . k_j
            sdb.soft_max(s, 1.0 / math.sqrt(c), out=s)
            o = sdb.mul_mat_transient(vt[i].view(c, lq), s)                     # o[i][c] = sum_j p_ij v_jc
            xv = x[i].view(lq, c)
            sdb.mul_mat(at.wo_lin, o, out=xv, chain=sdb.Chain().add(at.bo).redirect(xv, True))
        return x

    # ------------------------------------------------------------ decode

    def decode(self, z):
        """z (N, h, w, 4) channels-last latent (as the sampler leaves it) -> (N, 8h, 8w, 3)."""
        pq_w, pq_b = self.post_quant
        # post_quant_conv(z / scale_factor): the 1x1 convolution is linear, so the scale rides in its chain.
        h = sdb.conv2d_nhwc(pq_w, z, chain=sdb.Chain().mul(self.inv_scale, [0, 0, 0, 0]).add(pq_b, [0, 0, 1, 0]))
        h = self._conv3(self.conv_in[0], self.conv_in[1], h)
        rb1, attn, rb2 = self.mid
        h = self._resblock(h, rb1)
        h = self._attention(h, attn)
        h = self._resblock(h, rb2)
        for blocks, upsample in self.up:
            for rb in blocks:
                h = self._resblock(h, rb)
            if upsample is not None:
                h = sdb.upscale_nearest_nhwc(h, 2)
                h = self._conv3(upsample[0], upsample[1], h)
        t = self._gn(h, self.norm_out, True)
        return self._conv3(self.conv_out[0], self.conv_out[1], t)

    def flops(self, batch: int, height: int, width: int) -> int:
        """Algorithmic FLOPs of one decode of a (height x width) latent in the reference's convention
        (profile.cc:65-81): 2 KH KW IC OC OH OW N for convolutions, 2 M N K for products (attention's
        two products as 4 d Lq Lk)."""
        c = self.cfg

        def conv(ic, oc, k, h, w):
            return 2 * k * k * ic * oc * h * w * batch

        def rb_flops(rb, h, w):
            f = conv(rb.cin, rb.cout, 3, h, w) + conv(rb.cout, rb.cout, 3, h, w)
            return f + (conv(rb.cin, rb.cout, 1, h, w) if rb.skip is not None else 0)

        h, w = height, width
        block_in = c.ch * c.ch_mult[-1]
        total = conv(c.z_channels, c.z_channels, 1, h, w) + conv(c.z_channels, block_in, 3, h, w)
        rb1, at, rb2 = self.mid
        lq = h * w
        total += rb_flops(rb1, h, w) + rb_flops(rb2, h, w)
        total += 4 * conv(at.c, at.c, 1, h, w) + 4 * at.c * lq * lq * batch
        for blocks, upsample in self.up:
            for rb in blocks:
                total += rb_flops(rb, h, w)
            if upsample is not None:
                h, w = 2 * h, 2 * w
                total += conv(blocks[-1].cout, blocks[-1].cout, 3, h, w)
        total += conv(self.conv_out[0].shape[1], c.out_channels, 3, h, w)
        return total
