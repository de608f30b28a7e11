"""The SD 1.x UNet and its Euler / classifier-free-guidance sampler on the library's kernels.

stable-diffusion.cpp builds the UNet as a ggml graph whose MUL_MAT, CONV_2D,
FLASH_ATTN_EXT, GROUP_NORM and NORM nodes the reference computes on the CPU
(hooks.cc:29-55).  Here the same network runs device-resident: every one of
those nodes is a call into libsdb (sdb.py), the element-wise nodes after them
ride in their chains (bias, time embedding, scale and shift, SiLU, residual),
and the graph's other nodes (concat, nearest upscale, timestep embedding) are
libsdb's glue kernels.  Activations are channels-last, (N, H, W, C), so the
transformer's tokens are the image's rows with no permutes.  Two fusions the
graph allows: every ResBlock's time-embedding projection is one GEMM over the
concatenated weights, and so is every cross-attention's K/V projection of the
(fixed) text context.

Two configurations of the same ldm UNetModel (the benchmark's):
  SD15: model channels 320, multipliers 1/2/4/4, 2 ResBlocks a level, a
        SpatialTransformer of depth 1 with 8 heads at the first three levels
        and in the middle, context dim 768;
  SDXL: multipliers 1/2/4, transformers of depth 0/2/10 (10 in the middle)
        with heads of 64 dims, context dim 2048, and the label embedding of
        the pooled text embedding and the size/crop conditioning (2816 inputs)
        added to the time embedding.
Both: GroupNorm 32 (eps 1e-5; 1e-6 in the transformers), LayerNorm eps 1e-5,
GEGLU feed-forward of 4C, linear proj_in / proj_out, nearest 2x upsampling.
Weights are random (the benchmark's random-init FP16 weights), drawn from one
seed on the device.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import sdb


@dataclass(frozen=True)
class UNetConfig:
    in_channels: int = 4
    out_channels: int = 4
    model_channels: int = 320
    channel_mult: tuple = (1, 2, 4, 4)
    num_res_blocks: int = 2
    attention_levels: tuple = (0, 1, 2)
    heads: int = 8
    context_dim: int = 768
    groups: int = 32
    time_dim_mult: int = 4
    transformer_depth: tuple = ()      # blocks of the transformer at each level (empty: 1 at attention_levels)
    mid_depth: int = 1
    head_dim: int = 0                  # dims of a head (0: `heads` heads of C / heads)
    adm_in_channels: int = 0           # inputs of the label embedding (SDXL: pooled text + size/crop)

    def depth(self, level: int) -> int:
        if self.transformer_depth:
            return self.transformer_depth[level]
        return 1 if level in self.attention_levels else 0

    def heads_of(self, channels: int) -> int:
        return channels // self.head_dim if self.head_dim else self.heads


SD15 = UNetConfig()
SDXL = UNetConfig(channel_mult=(1, 2, 4), attention_levels=(1, 2), transformer_depth=(0, 2, 10), mid_depth=10,
                  head_dim=64, context_dim=2048, adm_in_channels=2816)


# ---------------------------------------------------------------- weights

class _Init:
    """Random FP16 weights and FP32 biases / norm parameters from one seed, on the device."""

    def __init__(self, device, seed: int):
        import torch

        self.torch = torch
        self.device = device
        self.gen = torch.Generator(device=device)
        self.gen.manual_seed(seed)
        self.params = 0

    def normal(self, shape, std, dtype, mean=0.0):
        t = self.torch.randn(*shape, generator=self.gen, device=self.device, dtype=self.torch.float32)
        t = t * std + mean
        self.params += t.numel()
        return t.to(dtype).contiguous()

    def conv(self, oc, ic, k):
        return self.normal((oc, ic, k, k), 1.0 / math.sqrt(ic * k * k), self.torch.float16)

    def linear(self, n, k):
        return self.normal((n, k), 1.0 / math.sqrt(k), self.torch.float16)

    def bias(self, n):
        return self.normal((n,), 0.02, self.torch.float32)

    def gamma(self, n):
        return self.normal((n,), 0.1, self.torch.float32, mean=1.0)

    def beta(self, n):
        return self.normal((n,), 0.1, self.torch.float32)


@dataclass
class ResBlock:
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
    emb_offset: int = 0       # columns of this block in the fused time-embedding projection


@dataclass
class TBlock:
    """One BasicTransformerBlock: self-attention, cross-attention on the context, GEGLU feed-forward."""
    ln1: tuple
    wqkv: object
    wo1: object
    bo1: object
    ln2: tuple
    wq2: object
    wo2: object
    bo2: object
    ln3: tuple
    wff1: object
    bff1: object
    wff2: object
    bff2: object
    kv_offset: int = 0        # columns of this block's K/V in the fused context projection
    wq: object = None         # wqkv's query rows, and its key and value rows (ToDo projects them apart):
    wkv: object = None        #   views made once, so that the weight store keeps one packing of each


@dataclass
class Transformer:
    c: int
    heads: int
    gn: tuple
    proj_in: object
    b_in: object
    blocks: list
    proj_out: object
    b_out: object


@dataclass
class Level:
    blocks: list = field(default_factory=list)   # (ResBlock, Transformer | None)
    down: tuple | None = None                    # (weight, bias)
    up: tuple | None = None


class UNet:
    """SD 1.x UNet on libsdb: forward(x (B, H, W, 4), timesteps (B,), context (B, 77, 768)) -> eps (B, H, W, 4)."""

    def __init__(self, config: UNetConfig = SD15, device="cuda", seed: int = 20261011):
        import torch

        self.torch = torch
        self.cfg = config
        self.device = torch.device(device)
        init = _Init(self.device, seed)
        c = config
        mc = c.model_channels
        td = mc * c.time_dim_mult
        self.time_dim = td
        self.t_w1, self.t_b1 = init.linear(td, mc), init.bias(td)
        self.t_w2, self.t_b2 = init.linear(td, td), init.bias(td)
        self.conv_in, self.conv_in_b = init.conv(mc, c.in_channels, 3), init.bias(mc)
        res_blocks: list[ResBlock] = []
        transformers: list[Transformer] = []

        def resblock(cin, cout):
            rb = ResBlock(cin, cout, (init.gamma(cin), init.beta(cin)), init.conv(cout, cin, 3), init.bias(cout),
                          (init.gamma(cout), init.beta(cout)), init.conv(cout, cout, 3), init.bias(cout))
            if cin != cout:
                rb.skip, rb.bskip = init.conv(cout, cin, 1), init.bias(cout)
            res_blocks.append(rb)
            return rb

        def transformer(ch, depth):
            if depth == 0:
                return None
            gn, proj_in, b_in = (init.gamma(ch), init.beta(ch)), init.linear(ch, ch), init.bias(ch)
            blocks = [TBlock((init.gamma(ch), init.beta(ch)), init.linear(3 * ch, ch), init.linear(ch, ch),
                             init.bias(ch), (init.gamma(ch), init.beta(ch)), init.linear(ch, ch), init.linear(ch, ch),
                             init.bias(ch), (init.gamma(ch), init.beta(ch)), init.linear(8 * ch, ch),
                             init.bias(8 * ch), init.linear(ch, 4 * ch), init.bias(ch)) for _ in range(depth)]
            for blk in blocks:
                blk.wq, blk.wkv = blk.wqkv[:ch], blk.wqkv[ch:]
            tr = Transformer(ch, c.heads_of(ch), gn, proj_in, b_in, blocks, init.linear(ch, ch), init.bias(ch))
            transformers.append(tr)
            return tr

        # Encoder.
        self.down: list[Level] = []
        chans = [mc]
        ch = mc
        for lvl, mult in enumerate(c.channel_mult):
            level = Level()
            for _ in range(c.num_res_blocks):
                rb = resblock(ch, mult * mc)
                ch = mult * mc
                level.blocks.append((rb, transformer(ch, c.depth(lvl))))
                chans.append(ch)
            if lvl != len(c.channel_mult) - 1:
                level.down = (init.conv(ch, ch, 3), init.bias(ch))
                chans.append(ch)
            self.down.append(level)
        # Middle.
        self.mid = (resblock(ch, ch), transformer(ch, c.mid_depth), resblock(ch, ch))
        # Decoder.
        self.up: list[Level] = []
        for lvl, mult in reversed(list(enumerate(c.channel_mult))):
            level = Level()
            for i in range(c.num_res_blocks + 1):
                skip = chans.pop()
                rb = resblock(ch + skip, mult * mc)
                ch = mult * mc
                level.blocks.append((rb, transformer(ch, c.depth(lvl))))
            if lvl != 0:
                level.up = (init.conv(ch, ch, 3), init.bias(ch))
            self.up.append(level)
        self.out_gn = (init.gamma(ch), init.beta(ch))
        self.conv_out, self.conv_out_b = init.conv(c.out_channels, ch, 3), init.bias(c.out_channels)
        if c.adm_in_channels:
            self.label_w1, self.label_b1 = init.linear(td, c.adm_in_channels), init.bias(td)
            self.label_w2, self.label_b2 = init.linear(td, td), init.bias(td)

        # Fused projections: all time-embedding projections, all context K/V projections.
        off = 0
        emb_w, emb_b = [], []
        for rb in res_blocks:
            rb.emb_offset = off
            off += rb.cout
            emb_w.append(init.linear(rb.cout, td))
            emb_b.append(init.bias(rb.cout))
        self.emb_w, self.emb_b = torch.cat(emb_w).contiguous(), torch.cat(emb_b).contiguous()
        off = 0
        kv_w = []
        for tr in transformers:
            for blk in tr.blocks:
                blk.kv_offset = off
                off += 2 * tr.c
                kv_w.append(init.linear(2 * tr.c, c.context_dim))
        self.kv_w = torch.cat(kv_w).contiguous() if kv_w else None
        self.res_blocks, self.transformers = res_blocks, transformers
        self.params = init.params
        # GroupNorm fused into the convolution or linear layer that reads it (sdb_conv2d_normed,
        # sdb_mul_mat_normed); False runs it as the reference's separate node (the same numbers).
        self.fuse_gn = True
        # LayerNorm fused into the linear layer that reads it (sdb_mul_mat_layer_normed); False: separate.
        self.fuse_ln = True

    # ------------------------------------------------------------ pieces

    def _gn(self, x, gn, eps, silu, out=None):
        ch = sdb.Chain().mul(gn[0], [0, 0, 1, 0]).add(gn[1], [0, 0, 1, 0])
        if silu:
            ch.silu()
        return sdb.group_norm_nhwc(x, self.cfg.groups, eps, out=out, chain=ch)

    def _gn_in(self, x, gn, eps, silu):
        """The GroupNorm (+ SiLU) of x as a prologue of the operation that reads it (fuse_gn): its
        statistics now, the normalisation as the next convolution or linear layer loads x."""
        return sdb.GroupNormIn(sdb.group_norm_stats(x, self.cfg.groups, eps), self.cfg.groups, gn[0], gn[1], silu)

    def _conv_gn(self, w, x, gn, eps, chain, out=None):
        """3x3 convolution of SiLU(GroupNorm(x)): fused (the statistics, then the convolution normalising
        its input as it reads it) or as the reference's separate nodes.  Fused where the convolution
        reads each input once (the direct path's split: images under 1024 positions); in front of a
        Winograd convolution, whose input transform reads each input (F + 2)^2 / F^2 = 2.25 times, the
        normalisation and SiLU run once as a pass of their own (measured faster there)."""
        winograd = w.shape[2] == 3 and x.shape[1] * x.shape[2] >= 1024
        if self.fuse_gn and not winograd:
            return sdb.conv2d_nhwc_normed(w, x, self._gn_in(x, gn, eps, True), (1, 1), (1, 1), out=out, chain=chain)
        return sdb.conv2d_nhwc(w, self._gn(x, gn, eps, True), (1, 1), (1, 1), out=out, chain=chain)

    def _resblock(self, x, rb: ResBlock, emb):
        emb_view = emb[:, rb.emb_offset:rb.emb_offset + rb.cout]
        h = self._conv_gn(rb.conv1, x, rb.gn1, 1e-5,
                          sdb.Chain().add(rb.b1, [0, 0, 1, 0]).add(emb_view, [0, 0, 1, emb.shape[1]]))
        if rb.skip is None:
            xs = (x.stride(2), x.stride(1), x.stride(3), x.stride(0))  # ggml order [W, H, C, N]
            return self._conv_gn(rb.conv2, h, rb.gn2, 1e-5, sdb.Chain().add(rb.b2, [0, 0, 1, 0]).add(x, list(xs)))
        out = sdb.conv2d_nhwc(rb.skip, x, chain=sdb.Chain().add(rb.bskip, [0, 0, 1, 0]))
        self._conv_gn(rb.conv2, h, rb.gn2, 1e-5, sdb.Chain().add(rb.b2, [0, 0, 1, 0]).redirect(out, True))
        return out

    def _ln(self, x, ln):
        return sdb.norm(x, 1e-5, chain=sdb.Chain().mul(ln[0]).add(ln[1]))

    def _ln_linear(self, w, x, ln, chain=None, gated=False):
        """The linear layer (or GEGLU) of LayerNorm(x): fused, the normalisation inside the layer's split of
        its rows (fuse_ln), or as the reference's separate NORM node."""
        if self.fuse_ln:
            return sdb.mul_mat_layer_normed(w, x, 1e-5, sdb.Chain().mul(ln[0]).add(ln[1]), chain=chain, gated=gated)
        h = self._ln(x, ln)
        return sdb.mul_mat_gated(w, h, chain=chain) if gated else sdb.mul_mat(w, h, chain=chain)

    def _transformer(self, x, tr: Transformer, ctx_kv):
        b, hh, ww, c = x.shape
        heads = tr.heads
        scale = 1.0 / math.sqrt(c // heads)
        if self.fuse_gn:
            t = sdb.mul_mat_normed(tr.proj_in, x.view(b, hh * ww, c), self._gn_in(x, tr.gn, 1e-6, False),
                                   chain=sdb.Chain().add(tr.b_in))
        else:
            n = self._gn(x, tr.gn, 1e-6, False)
            t = sdb.mul_mat(tr.proj_in, n.view(b, hh * ww, c), chain=sdb.Chain().add(tr.b_in))
        # ToDo (the reference's stable-diffusion.cpp patch 0004): self-attention's keys and values from
        # every f-th token of every f-th row when the tuning asks for it on a grid this large.
        f = sdb.token_downsampling(ww, hh)
        for blk in tr.blocks:
            # Self-attention.
            if f > 1:
                h1 = self._ln(t, blk.ln1)
                q = sdb.mul_mat(blk.wq, h1)
                kv = sdb.mul_mat(blk.wkv, sdb.coarser_tokens(h1, ww, hh, f))
                a = sdb.attention_heads(q, kv[:, :, :c], kv[:, :, c:], heads, heads, scale)
            else:
                qkv = self._ln_linear(blk.wqkv, t, blk.ln1)
                a = sdb.attention_heads(qkv[:, :, :c], qkv[:, :, c:2 * c], qkv[:, :, 2 * c:], heads, heads, scale)
            sdb.mul_mat(blk.wo1, a, out=t, chain=sdb.Chain().add(blk.bo1).redirect(t, True))
            # Cross-attention on the text context.
            q2 = self._ln_linear(blk.wq2, t, blk.ln2)
            kv = ctx_kv[:, :, blk.kv_offset:blk.kv_offset + 2 * c]
            a2 = sdb.attention_heads(q2, kv[:, :, :c], kv[:, :, c:], heads, heads, scale)
            sdb.mul_mat(blk.wo2, a2, out=t, chain=sdb.Chain().add(blk.bo2).redirect(t, True))
            # GEGLU feed-forward.
            g = self._ln_linear(blk.wff1, t, blk.ln3, chain=sdb.Chain().add(blk.bff1), gated=True)
            sdb.mul_mat(blk.wff2, g, out=t, chain=sdb.Chain().add(blk.bff2).redirect(t, True))
        # Back to the image, plus the block's input.
        xv = x.view(b, hh * ww, c)
        sdb.mul_mat(tr.proj_out, t, out=xv, chain=sdb.Chain().add(tr.b_out).redirect(xv, True))
        return x

    # ------------------------------------------------------------ forward

    def embed(self, timesteps, y=None):
        """SiLU(time_embed(timestep_embedding(t)) [+ label_emb(y)]) (B, 4 * model_channels), then every
        ResBlock's projection.  y (B, adm_in_channels): SDXL's pooled text embedding and size/crop
        conditioning."""
        mc = self.cfg.model_channels
        te = sdb.timestep_embedding(timesteps, mc)
        e1 = sdb.mul_mat(self.t_w1, te, chain=sdb.Chain().add(self.t_b1).silu())
        ch = sdb.Chain().add(self.t_b2)
        if self.cfg.adm_in_channels:
            l1 = sdb.mul_mat(self.label_w1, y, chain=sdb.Chain().add(self.label_b1).silu())
            l2 = sdb.mul_mat(self.label_w2, l1, chain=sdb.Chain().add(self.label_b2))
            ch.add(l2)
        e2 = sdb.mul_mat(self.t_w2, e1, chain=ch.silu())
        return sdb.mul_mat(self.emb_w, e2, chain=sdb.Chain().add(self.emb_b))

    def context_kv(self, context):
        """Every cross-attention's K and V of the context (B, 77, sum of 2C)."""
        return sdb.mul_mat(self.kv_w, context)

    def forward(self, x, timesteps, context, ctx_kv=None, y=None):
        emb = self.embed(timesteps, y)
        if ctx_kv is None:
            ctx_kv = self.context_kv(context)
        h = sdb.conv2d_nhwc(self.conv_in, x, (1, 1), (1, 1), chain=sdb.Chain().add(self.conv_in_b, [0, 0, 1, 0]))
        hs = [h]
        for level in self.down:
            for rb, tr in level.blocks:
                h = self._resblock(h, rb, emb)
                if tr is not None:
                    h = self._transformer(h, tr, ctx_kv)
                hs.append(h)
            if level.down is not None:
                h = sdb.conv2d_nhwc(level.down[0], h, (2, 2), (1, 1),
                                    chain=sdb.Chain().add(level.down[1], [0, 0, 1, 0]))
                hs.append(h)
        rb1, tr, rb2 = self.mid
        h = self._resblock(h, rb1, emb)
        h = self._transformer(h, tr, ctx_kv)
        h = self._resblock(h, rb2, emb)
        for level in self.up:
            for rb, tr in level.blocks:
                h = sdb.concat_channels_nhwc(h, hs.pop())
                h = self._resblock(h, rb, emb)
                if tr is not None:
                    h = self._transformer(h, tr, ctx_kv)
            if level.up is not None:
                h = sdb.upscale_nearest_nhwc(h, 2)
                h = sdb.conv2d_nhwc(level.up[0], h, (1, 1), (1, 1), chain=sdb.Chain().add(level.up[1], [0, 0, 1, 0]))
        return self._conv_gn(self.conv_out, h, self.out_gn, 1e-5, sdb.Chain().add(self.conv_out_b, [0, 0, 1, 0]))

    def flops(self, batch: int, height: int, width: int, context_len: int = 77) -> int:
        """Algorithmic FLOPs of one forward in the reference's convention (profile.cc:65-81):
        2 KH KW IC OC OH OW N for convolutions, 2 M N K for linear layers, 4 d h Lq Lk for attention."""
        c = self.cfg
        total = 0
        hw = [(height, width)]
        for lvl in range(1, len(c.channel_mult)):
            h, w = hw[-1]
            hw.append(((h + 1) // 2, (w + 1) // 2))

        def conv(ic, oc, k, h, w):
            return 2 * k * k * ic * oc * h * w * batch

        def tr_flops(tr, h, w):
            ch = tr.c
            L = h * w
            f = 2 * L * ch * ch * 2 * batch                    # proj_in, proj_out
            blk = 2 * L * ch * 3 * ch * batch + 4 * ch * L * L * batch + 2 * L * ch * ch * batch
            blk += 2 * L * ch * ch * batch + 4 * ch * L * context_len * batch + 2 * L * ch * ch * batch
            blk += 2 * batch * context_len * c.context_dim * 2 * ch    # K/V of the context
            blk += 2 * L * ch * 8 * ch * batch + 2 * L * 4 * ch * ch * batch
            return f + len(tr.blocks) * blk

        def rb_flops(rb, h, w):
            f = conv(rb.cin, rb.cout, 3, h, w) + conv(rb.cout, rb.cout, 3, h, w)
            if rb.skip is not None:
                f += conv(rb.cin, rb.cout, 1, h, w)
            return f + 2 * batch * self.time_dim * rb.cout

        mc = c.model_channels
        td = self.time_dim
        total += 2 * batch * (mc * td + td * td)
        if c.adm_in_channels:
            total += 2 * batch * (c.adm_in_channels * td + td * td)
        total += conv(c.in_channels, mc, 3, height, width)
        for lvl, level in enumerate(self.down):
            h, w = hw[lvl]
            for rb, tr in level.blocks:
                total += rb_flops(rb, h, w) + (tr_flops(tr, h, w) if tr else 0)
            if level.down is not None:
                ch = level.blocks[-1][0].cout
                total += conv(ch, ch, 3, *hw[lvl + 1])
        h, w = hw[-1]
        rb1, tr, rb2 = self.mid
        total += rb_flops(rb1, h, w) + tr_flops(tr, h, w) + rb_flops(rb2, h, w)
        for i, level in enumerate(self.up):
            lvl = len(c.channel_mult) - 1 - i
            h, w = hw[lvl]
            for rb, tr in level.blocks:
                total += rb_flops(rb, h, w) + (tr_flops(tr, h, w) if tr else 0)
            if level.up is not None:
                ch = level.blocks[-1][0].cout
                total += conv(ch, ch, 3, *hw[lvl - 1])
        total += conv(mc, c.out_channels, 3, height, width)
        return total


# ---------------------------------------------------------------- sampler

def discrete_sigmas(steps: int) -> list[float]:
    """The discrete sigmas of SD 1.x's scaled-linear schedule (1000 steps, beta 0.00085 .. 0.012), `steps`
    of them evenly spaced in timestep from 999 to 0, then 0 -- stable-diffusion.cpp's default schedule."""
    betas = [(math.sqrt(0.00085) + (math.sqrt(0.012) - math.sqrt(0.00085)) * i / 999) ** 2 for i in range(1000)]
    alphas_cum, acc = [], 1.0
    for b in betas:
        acc *= 1.0 - b
        alphas_cum.append(acc)
    all_sigmas = [math.sqrt((1 - a) / a) for a in alphas_cum]
    out = []
    for i in range(steps):
        t = 999.0 - 999.0 * i / max(1, steps - 1)
        lo = int(math.floor(t))
        hi = min(lo + 1, 999)
        w = t - lo
        log_sigma = (1 - w) * math.log(all_sigmas[lo]) + w * math.log(all_sigmas[hi])
        out.append(math.exp(log_sigma))
    out.append(0.0)
    return out


def sigma_to_t(sigma: float) -> float:
    """The (fractional) timestep of a sigma on the same schedule, by log-sigma interpolation."""
    betas = [(math.sqrt(0.00085) + (math.sqrt(0.012) - math.sqrt(0.00085)) * i / 999) ** 2 for i in range(1000)]
    acc, logs = 1.0, []
    for b in betas:
        acc *= 1.0 - b
        logs.append(math.log(math.sqrt((1 - acc) / acc)))
    ls = math.log(max(sigma, 1e-10))
    if ls <= logs[0]:
        return 0.0
    for i in range(999):
        if logs[i] <= ls <= logs[i + 1]:
            return i + (ls - logs[i]) / (logs[i + 1] - logs[i])
    return 999.0


class Sampler:
    """Euler sampling with classifier-free guidance of `images` images at once: per step one UNet forward
    on the batch [the images unconditional, the images conditional] and one fused guidance + Euler update
    (sdb_euler_cfg_step, whose halves are those two).  The per-step forward is captured once as a CUDA
    graph and replayed."""

    def __init__(self, unet: UNet, height: int = 64, width: int = 64, steps: int = 20, cfg_scale: float = 7.0,
                 context_len: int = 77, images: int = 1):
        torch = unet.torch
        self.unet, self.steps, self.cfg_scale, self.images = unet, steps, cfg_scale, images
        dev = unet.device
        c = unet.cfg
        self.sigmas = discrete_sigmas(steps)
        self.x = torch.zeros(images, height, width, c.in_channels, device=dev)
        self.x_in = torch.zeros(2 * images, height, width, c.in_channels, device=dev)
        self.t = torch.zeros(2 * images, device=dev)
        self.context = torch.zeros(2 * images, context_len, c.context_dim, device=dev)
        self.eps = None
        self.graph = None

    def _forward(self):
        ctx_kv = self.unet.context_kv(self.context)
        self.eps = self.unet.forward(self.x_in, self.t, self.context, ctx_kv)
        return self.eps

    def capture(self, warmup: int = 2):
        """Runs the forward eagerly (the library's workspace and weight store settle), then captures it."""
        torch = self.unet.torch
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._forward()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        # The same stream as the warm-up: the library's workspace is kept per stream.
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self._forward()
        torch.cuda.synchronize()

    def step_forward(self):
        """One UNet forward on the current inputs (graph replay when captured)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._forward()
        return self.eps

    def set_step(self, i: int):
        sigma = self.sigmas[i]
        self.t.fill_(sigma_to_t(sigma))
        self.x_in.view(2, *self.x.shape).copy_(self.x.unsqueeze(0).expand(2, *self.x.shape) /
                                               math.sqrt(sigma * sigma + 1.0))

    def sample(self, latent, context):
        """latent (images, H, W, 4) N(0, 1), context (2 images, 77, 768) [the images' unconditional, their
        conditional] -> the final latents."""
        self.x.copy_(latent * self.sigmas[0])
        self.context.copy_(context)
        for i in range(self.steps):
            self.set_step(i)
            eps = self.step_forward()
            sig, nxt = self.sigmas[i], self.sigmas[i + 1]
            sdb.euler_cfg_step(eps, self.x, None, self.cfg_scale, sig, nxt, 0.0)
        return self.x


# ---------------------------------------------------------------- guidance split over a GPU pair

def pair_groups(dist, world: int):
    """The process groups of the rank pairs (0, 1), (2, 3), ...: every rank creates every group, in the same
    order, as torch.distributed requires."""
    return [dist.new_group([2 * p, 2 * p + 1]) for p in range(world // 2)]


def gather_guidance(dist, group, eps_half, eps_full):
    """The two halves' eps meet: eps_full [2, ...] = [the pair's lower rank's, the higher rank's] -- the
    unconditional half on the lower rank, the conditional on the higher.  One all-gather of the pair (NCCL
    over NVLink between GPUs; 64 KiB an image for SD 1.5's 64 x 64 x 4 latent)."""
    dist.all_gather_into_tensor(eps_full, eps_half, group=group)
    return eps_full


class PairSampler:
    """Euler sampling with classifier-free guidance split over a pair of ranks: each runs the UNet on its
    half of the guidance batch (the lower rank unconditional, the higher conditional; batch 1 each), the
    halves' eps are gathered over the pair (gather_guidance), and both ranks take the same guidance + Euler
    update, so their latents stay identical.  The half forward is captured once as a CUDA graph; the
    all-gather runs on the same stream between replays."""

    def __init__(self, unet: UNet, dist, group, half: int, height: int = 64, width: int = 64, steps: int = 20,
                 cfg_scale: float = 7.0, context_len: int = 77):
        torch = unet.torch
        self.unet, self.dist, self.group, self.half = unet, dist, group, half
        self.steps, self.cfg_scale = steps, cfg_scale
        dev = unet.device
        c = unet.cfg
        self.sigmas = discrete_sigmas(steps)
        self.x = torch.zeros(1, height, width, c.in_channels, device=dev)
        self.x_in = torch.zeros(1, height, width, c.in_channels, device=dev)
        self.t = torch.zeros(1, device=dev)
        self.context = torch.zeros(1, context_len, c.context_dim, device=dev)
        self.eps_full = torch.zeros(2, height, width, c.in_channels, device=dev)
        self.eps = None
        self.graph = None
        self.stream = None

    def _forward(self):
        self.eps = self.unet.forward(self.x_in, self.t, self.context, self.unet.context_kv(self.context))
        return self.eps

    def capture(self, warmup: int = 2):
        torch = self.unet.torch
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._forward()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            self._forward()
        torch.cuda.synchronize()
        self.stream = s

    def set_step(self, i: int):
        sigma = self.sigmas[i]
        self.t.fill_(sigma_to_t(sigma))
        self.x_in.copy_(self.x / math.sqrt(sigma * sigma + 1.0))

    def step(self, i: int):
        """One sampler step: the half forward, the pair's all-gather, the guidance + Euler update, the
        next step's model input."""
        torch = self.unet.torch
        with torch.cuda.stream(self.stream):
            if self.graph is not None:
                self.graph.replay()
            else:
                self._forward()
            gather_guidance(self.dist, self.group, self.eps, self.eps_full)
            sig, nxt = self.sigmas[i], self.sigmas[i + 1]
            sdb.euler_cfg_step(self.eps_full, self.x, None, self.cfg_scale, sig, nxt, 0.0, stream=self.stream)
            self.x_in.copy_(self.x / math.sqrt(nxt * nxt + 1.0))

