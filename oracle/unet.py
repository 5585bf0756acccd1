"""CPU restatement of the reference's SD 1.x UNet forward (fp32), built on the oracle kernels.

TEST INFRASTRUCTURE ONLY (the checker for the GPU step and the timed CPU baseline).
Follows rhi-zone/sketchpad:
  crates/sketchpad-unet/src/unet_sd.rs:108-232  UNet::new (channel bookkeeping restated below)
  crates/sketchpad-unet/src/unet_sd.rs:235-272  UNet::forward
  crates/sketchpad-unet/src/unet_sd.rs:341-376, :414-418, :470-483  Down/Mid/Up block forwards
  crates/sketchpad-unet/src/blocks.rs:27-39, :123-150, :213-231, :292-305, :370-410, :446-458,
  :491, :526-535 (timestep embedding, ResBlock, SpatialTransformer, TransformerBlock,
  CrossAttention, FeedForward, Downsample, Upsample)
Parameters are looked up by the names sketchpad_b200.unet.make_unet_params gives them, so the
oracle and the GPU step run on identical synthetic weights.
"""
from __future__ import annotations

import math

import numpy as np

from . import activation, attention, conv2d, groupnorm_act, layernorm, linear_kn


class OracleUNet:
    def __init__(self, params, model_channels=320, channel_mult=(1, 2, 4, 4), num_heads=8,
                 head_dim=40, in_channels=4, out_channels=4):
        self.P = {k: np.ascontiguousarray(v, np.float32) for k, v in params.items()}
        self.ch, self.mult = model_channels, tuple(channel_mult)
        self.heads, self.hd = num_heads, head_dim
        half = model_channels // 2
        self.freqs = np.array([math.exp(-(i / half) * math.log(10000.0)) for i in range(half)],
                              np.float32)

    # ---- layers -------------------------------------------------------------------------
    def lin(self, x, name, bias=True):
        b = self.P.get(name + ".bias") if bias else None
        return linear_kn(x, self.P[name + ".weight"], b)

    def conv(self, x, name, stride=1):
        w = self.P[name + ".weight"]
        return conv2d(x, w, self.P[name + ".bias"], stride, w.shape[-1] // 2)

    def gn(self, x, name, silu):
        return groupnorm_act(x, self.P[name + ".weight"], self.P[name + ".bias"], 32, 1e-5, silu)

    def ln(self, x, name):
        return layernorm(x, self.P[name + ".weight"], self.P[name + ".bias"], 1e-5)

    # ---- blocks -------------------------------------------------------------------------
    def resblock(self, x, temb, p):  # blocks.rs:123-150
        residual = self.conv(x, p + ".skip_conv") if (p + ".skip_conv.weight") in self.P else x
        h = self.gn(x, p + ".norm1", True)
        h = self.conv(h, p + ".conv1")
        t = self.lin(activation(temb, "silu"), p + ".time_emb_proj")
        h = h + t[:, :, None, None]
        h = self.gn(h, p + ".norm2", True)
        h = self.conv(h, p + ".conv2")
        return h + residual

    def cross_attention(self, x, p, ctx):  # blocks.rs:370-410
        ctx = x if ctx is None else ctx
        b, s, _ = x.shape
        c = ctx.shape[1]
        q = self.lin(x, p + ".to_q", bias=False).reshape(b, s, self.heads, self.hd).transpose(0, 2, 1, 3)
        k = self.lin(ctx, p + ".to_k", bias=False).reshape(b, c, self.heads, self.hd).transpose(0, 2, 1, 3)
        v = self.lin(ctx, p + ".to_v", bias=False).reshape(b, c, self.heads, self.hd).transpose(0, 2, 1, 3)
        o = attention(q, k, v, variant=0)
        o = o.transpose(0, 2, 1, 3).reshape(b, s, self.heads * self.hd)
        return self.lin(o, p + ".to_out")

    def transformer_block(self, x, ctx, p):  # blocks.rs:292-305
        x = x + self.cross_attention(self.ln(x, p + ".norm1"), p + ".attn1", None)
        x = x + self.cross_attention(self.ln(x, p + ".norm2"), p + ".attn2", ctx)
        hdn = self.lin(self.ln(x, p + ".norm3"), p + ".ff.net_0")
        half = hdn.shape[-1] // 2
        hdn = hdn[..., :half] * activation(hdn[..., half:], "gelu")
        return x + self.lin(hdn, p + ".ff.net_2")

    def spatial_transformer(self, x, ctx, p):  # blocks.rs:213-231
        b, _, h, w = x.shape
        residual = x
        y = self.gn(x, p + ".norm", False)
        y = self.conv(y, p + ".proj_in")
        inner = y.shape[1]
        y = y.reshape(b, inner, h * w).transpose(0, 2, 1)
        y = self.transformer_block(np.ascontiguousarray(y), ctx, p + ".tb0")
        y = y.transpose(0, 2, 1).reshape(b, inner, h, w)
        return self.conv(np.ascontiguousarray(y), p + ".proj_out") + residual

    @staticmethod
    def upsample_nearest(x):  # blocks.rs:526-535
        return x.repeat(2, axis=2).repeat(2, axis=3)

    # ---- UNet::forward --------------------------------------------------------------------
    def forward(self, x, timesteps, context):
        x = np.ascontiguousarray(x, np.float32)
        context = np.ascontiguousarray(context, np.float32)
        args = np.asarray(timesteps, np.float32)[:, None] * self.freqs[None, :]
        temb = np.concatenate([np.sin(args), np.cos(args)], axis=1).astype(np.float32)
        temb = self.lin(temb, "time_embed_0")
        temb = self.lin(activation(temb, "silu"), "time_embed_2")
        h = self.conv(x, "conv_in")
        skips = [h]
        n = len(self.mult)
        for level in range(n):  # down blocks: levels 0-2 carry attention, the last no downsample
            p = f"down{level}"
            att, last = level < 3, level == n - 1
            h = self.resblock(h, temb, p + ".res1")
            if att:
                h = self.spatial_transformer(h, context, p + ".attn1")
            skips.append(h)
            h = self.resblock(h, temb, p + ".res2")
            if att:
                h = self.spatial_transformer(h, context, p + ".attn2")
            skips.append(h)
            if not last:
                h = self.conv(h, p + ".downsample", stride=2)
                skips.append(h)
        h = self.resblock(h, temb, "mid.res1")
        h = self.spatial_transformer(h, context, "mid.attn")
        h = self.resblock(h, temb, "mid.res2")
        ui = 0
        for level in range(n):  # reversed levels; attention except the deepest level
            att, last = level > 0, level == n - 1
            for i in range(3):
                p = f"up{ui}"
                h = np.concatenate([h, skips.pop()], axis=1)
                h = self.resblock(h, temb, p + ".res")
                if att:
                    h = self.spatial_transformer(h, context, p + ".attn")
                if i == 2 and not last:
                    h = self.conv(self.upsample_nearest(h), p + ".upsample")
                ui += 1
        h = self.gn(h, "norm_out", True)
        return self.conv(h, "conv_out")

    __call__ = forward
