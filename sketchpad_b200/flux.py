"""Flux-shaped MMDiT denoise step with Q8_0 weights on the B200 kernels.

Follows rhi-zone/sketchpad crates/sketchpad-dit/src/flux.rs:
  :60-96     FluxConfig::flux_dev (hidden 3072, 24 heads x 128, 19 double + 38 single blocks,
             text_dim 4096, time_dim 256, mlp_ratio 4); max_seq_len must cover 4608 tokens
             for the single blocks (the reference's default 4096 cache would be sliced past)
  :199-247   timestep_freqs / TimestepEmbedding::forward_scalar
  :325-422   FluxAttention::forward (qkv -> RoPE on the stream's own q,k -> K/V = cat(self,
             other stream through the SAME qkv, no RoPE) -> softmax(QK^T/sqrt(d))V -> proj)
  :450-517   FluxDoubleBlock::forward (image stream first; the text stream attends to the
             UPDATED image tokens)
  :573-607   FluxSingleBlock::forward (one gate for both residual branches)
  :620-636   FinalLayer, :686-741 Flux::forward
  crates/sketchpad-core/src/rope.rs:60-170   1-D interleaved-pair RoPE, theta 10000
  crates/sketchpad-core/src/glu.rs:91-96     SwiGLU: down(silu(gate(x)) * up(x)), biased
  crates/sketchpad-core/src/dit.rs:299-345   PatchEmbed / unpatchify
Every Linear is a Q8_0 GpuQuantizedLinear (fused dequant-GEMM); attention is the tcgen05
flash kernel; LayerNorm is the unbiased kernel.  RoPE, modulation and SwiGLU gating are torch
element-wise glue.  Weights: int8 ~ U[-127,127], f16 block scale ~ U(0.001, 0.02), biases
~ N(0, 0.02) (the config's synthetic init; the values blow activations up over 57 blocks,
so whole-model numbers are timing-only -- parity is checked per block).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from .attention import flash_attention
from .layernorm import layer_norm_modulate
from .quantized_matmul import (GLU_SWIGLU, GpuQuantizedLinear, RopeEpilogue, interleave_rows,
                               rope_pair_table)


@dataclass(frozen=True)
class FluxConfig:
    in_channels: int = 16
    patch_size: int = 2
    hidden_size: int = 3072
    num_heads: int = 24
    num_double_blocks: int = 19
    num_single_blocks: int = 38
    text_dim: int = 4096
    time_dim: int = 256
    guidance_dim: int = 256
    max_seq_len: int = 4608
    mlp_ratio: float = 4.0
    # synthetic Q8_0 block scales ~ U(lo, hi) (config 4: 0.001 .. 0.02)
    weight_scale: tuple = (0.001, 0.02)

    @property
    def head_dim(self):
        return self.hidden_size // self.num_heads

    @property
    def intermediate(self):
        return int(self.hidden_size * self.mlp_ratio)


def flux_timestep_freqs(dim: int) -> np.ndarray:
    """flux.rs:199-207 (emb_scale = -ln(2) / (half - 1), as the reference writes it)."""
    half = dim // 2
    emb_scale = np.float32(-math.log(2.0)) / np.float32(half - 1)
    return np.exp(emb_scale * np.arange(half, dtype=np.float32)).astype(np.float32)


def rope_tables(head_dim: int, seq_len: int, base: float = 10000.0):
    """rope.rs:60-94: cos/sin [seq, head_dim], each frequency repeated for its pair."""
    half = head_dim // 2
    inv = np.array([1.0 / (base ** ((2 * i) / head_dim)) for i in range(half)], np.float32)
    ang = np.arange(seq_len, dtype=np.float32)[:, None] * inv[None, :]
    cos = np.repeat(np.cos(ang), 2, axis=1).astype(np.float32)
    sin = np.repeat(np.sin(ang), 2, axis=1).astype(np.float32)
    return cos, sin


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """rope.rs:145-170: x*cos + rotate_half(x)*sin, rotate_half([x0,x1,..]) = [-x1,x0,..]."""
    S = x.shape[2]
    x2 = x.unflatten(-1, (-1, 2))
    rot = torch.stack((-x2[..., 1], x2[..., 0]), dim=-1).flatten(-2)
    return x * cos[:S] + rot * sin[:S]


def _q8_linear(rng_seed: int, n: int, k: int, device, bias=True, scale_range=(0.001, 0.02)):
    """A Q8_0 Linear [n out, k in] with the config's synthetic weights, drawn on the device:
    int8 ~ U[-127, 127], f16 block scale ~ U(scale_range), bias ~ N(0, 0.02)."""
    g = torch.Generator(device=device).manual_seed(rng_seed)
    q = torch.randint(-127, 128, (n, k), generator=g, device=device, dtype=torch.int32).to(torch.int8)
    lo, hi = scale_range
    s = (torch.rand((k // 32, n), generator=g, device=device) * (hi - lo) + lo).to(torch.float16)
    b = (torch.randn(n, generator=g, device=device) * 0.02).to(torch.bfloat16) if bias else None
    return GpuQuantizedLinear(q, s.view(torch.int16), n, k, torch.bfloat16, b)


class _Attn:
    def __init__(self, seed, cfg: FluxConfig, device):
        h = cfg.hidden_size
        self.qkv = _q8_linear(seed, 3 * h, h, device, scale_range=cfg.weight_scale)
        self.proj = _q8_linear(seed + 1, h, h, device, scale_range=cfg.weight_scale)
        # rows [h, 3h) of the qkv weight produce k and v: the cross stream needs only those
        self.kv = GpuQuantizedLinear(self.qkv.q[h:], self.qkv.scale[:, h:].contiguous(), 2 * h, h,
                                     torch.bfloat16,
                                     self.qkv.bias[h:])
        self.H, self.D = cfg.num_heads, cfg.head_dim
        # a dict here receives this attention's bf16 inputs (q after RoPE, joint k and v) on
        # every forward: parity tests feed them to the oracle to check the later stages alone
        self.record = None

    def forward(self, x, cos, sin, cross=None, gate=None, residual=None, out=None):
        """proj(attention(x)); with gate [h] and residual: residual + gate * proj(...), the
        gated residual add done in the projection's epilogue."""
        b, s, _ = x.shape
        if _epilogue_fusable(x):
            return self._forward_joint(x, cos, sin, cross, gate, residual, out)
        qkv = self.qkv(x).view(b, s, 3, self.H, self.D)
        q = apply_rope(qkv[:, :, 0].transpose(1, 2), cos, sin)
        k = apply_rope(qkv[:, :, 1].transpose(1, 2), cos, sin)
        v = qkv[:, :, 2].transpose(1, 2)
        if cross is not None:
            c = cross.shape[1]
            kv = self.kv(cross).view(b, c, 2, self.H, self.D)
            k = torch.cat([k, kv[:, :, 0].transpose(1, 2)], dim=2)
            v = torch.cat([v, kv[:, :, 1].transpose(1, 2)], dim=2)
        o = torch.empty((b, s, self.H, self.D), dtype=x.dtype, device=x.device)
        flash_attention(q, k, v, out=o.transpose(1, 2))
        return self.proj(o.view(b, s, self.H * self.D), out=out, gate=gate, residual=residual)

    def _forward_joint(self, x, cos, sin, cross, gate, residual, out):
        """One prompt: the qkv GEMM writes q, k, v with RoPE applied in its epilogue into a
        joint [s + c, 3h] buffer whose last c rows receive the cross stream's k, v from the
        kv GEMM, so attention reads K = [k_self; k_cross] and V likewise in place (no
        rotation or concatenation passes)."""
        _, s, h = x.shape
        c = cross.shape[1] if cross is not None else 0
        buf = torch.empty((1, s + c, 3 * h), dtype=x.dtype, device=x.device)
        self.qkv(x, out=buf[:, :s], rope=RopeEpilogue(_rope_pairs(cos, sin), 2 * h, self.D))
        if c:
            self.kv(cross, out=buf[:, s:, h:])
        if self.record is not None:
            self.record.update(q=buf[:, :s, :h].clone(), k=buf[:, :, h:2 * h].clone(),
                               v=buf[:, :, 2 * h:].clone())
        heads = lambda t: t.unflatten(-1, (self.H, self.D)).transpose(1, 2)  # noqa: E731
        o = torch.empty((1, s, self.H, self.D), dtype=x.dtype, device=x.device)
        flash_attention(heads(buf[:, :s, :h]), heads(buf[:, :, h:2 * h]), heads(buf[:, :, 2 * h:]),
                        out=o.transpose(1, 2))
        return self.proj(o.view(1, s, h), out=out, gate=gate, residual=residual)


class _SwiGlu:
    def __init__(self, seed, cfg: FluxConfig, device):
        h, i = cfg.hidden_size, cfg.intermediate
        gate = _q8_linear(seed, i, h, device, scale_range=cfg.weight_scale)
        up = _q8_linear(seed + 1, i, h, device, scale_range=cfg.weight_scale)
        # gate and up share x: one GEMM over their rows interleaved (gate j, up j), whose
        # epilogue forms silu(gate) * up (no [M, 2I] intermediate)
        self.gate_up = GpuQuantizedLinear(interleave_rows(gate.q, up.q),
                                          interleave_rows(gate.scale, up.scale, dim=1),
                                          2 * i, h, torch.bfloat16,
                                          interleave_rows(gate.bias, up.bias))
        self.down = _q8_linear(seed + 2, h, i, device, scale_range=cfg.weight_scale)
        self.i = i

    def forward(self, x, gate=None, residual=None, out=None):
        # silu(gate) * up in gate_up's epilogue; the optional gated residual add in down's
        return self.down(self.gate_up(x, glu=GLU_SWIGLU), out=out, gate=gate, residual=residual)


def _ln(x, scale=None, shift=None):
    # LayerNorm::new(hidden) (gamma 1, beta 0, unbiased variance, layernorm.rs:63-73), with
    # the blocks' `(1 + scale) * x + shift` modulation fused when scale / shift are given
    return layer_norm_modulate(x, scale, shift, 1e-5, True)


def _rope_pairs(cos, sin):
    """The f32 (cos, sin) pair table of the RoPE epilogue for these [positions, head_dim]
    tables: the one FluxB200 attached (built from f32 angles), else derived once and kept on
    the `cos` tensor."""
    t = getattr(cos, "_sp_rope_pairs", None)
    if t is None:
        t = rope_pair_table(cos, sin)
        cos._sp_rope_pairs = t
    return t


def _epilogue_fusable(r):
    # the GEMM epilogue takes one gate vector and a contiguous bf16 residual
    return r.shape[0] == 1 and r.dtype == torch.bfloat16 and r.is_contiguous()


def _gated_add(r, gate, branch, in_place=False):
    """r + gate * branch(): `gate` is the modulation's [b, 1, h] slice.  For one prompt
    (b == 1) the add runs in the branch's last GEMM epilogue (in place on `r` when
    `in_place`, which callers use only on a tensor this block created); otherwise as
    torch element-wise ops."""
    if _epilogue_fusable(r):
        return branch(gate=gate.reshape(-1), residual=r, out=r if in_place else None)
    return r + gate * branch()


class FluxDoubleBlockB200:
    def __init__(self, seed, cfg: FluxConfig, device):
        h = cfg.hidden_size
        self.img_attn, self.txt_attn = _Attn(seed, cfg, device), _Attn(seed + 10, cfg, device)
        self.img_ffn, self.txt_ffn = _SwiGlu(seed + 20, cfg, device), _SwiGlu(seed + 30, cfg, device)
        self.modulation = _q8_linear(seed + 40, 6 * h, h, device, scale_range=cfg.weight_scale)
        self.h = h

    def forward(self, img, txt, cond, cos, sin):
        b = img.shape[0]
        m = self.modulation(cond).view(b, 1, 6, self.h)
        shift, scale, gate = m[:, :, 0], m[:, :, 1], m[:, :, 2]
        x = _ln(img, scale, shift)
        img = _gated_add(img, gate, lambda **kw: self.img_attn.forward(x, cos, sin, txt, **kw))
        img = _gated_add(img, gate, lambda **kw: self.img_ffn.forward(_ln(img), **kw), True)
        shift, scale, gate = m[:, :, 3], m[:, :, 4], m[:, :, 5]
        x = _ln(txt, scale, shift)
        txt = _gated_add(txt, gate, lambda **kw: self.txt_attn.forward(x, cos, sin, img, **kw))
        txt = _gated_add(txt, gate, lambda **kw: self.txt_ffn.forward(_ln(txt), **kw), True)
        return img, txt


class FluxSingleBlockB200:
    def __init__(self, seed, cfg: FluxConfig, device):
        h = cfg.hidden_size
        self.attn = _Attn(seed, cfg, device)
        self.ffn = _SwiGlu(seed + 20, cfg, device)
        self.modulation = _q8_linear(seed + 40, 3 * h, h, device, scale_range=cfg.weight_scale)
        self.h = h

    def forward(self, x, cond, cos, sin):
        b = x.shape[0]
        m = self.modulation(cond).view(b, 1, 3, self.h)
        shift, scale, gate = m[:, :, 0], m[:, :, 1], m[:, :, 2]
        xn = _ln(x, scale, shift)
        x = _gated_add(x, gate, lambda **kw: self.attn.forward(xn, cos, sin, **kw))
        return _gated_add(x, gate, lambda **kw: self.ffn.forward(_ln(x), **kw), True)


class FluxB200:
    """Flux::forward (flux.rs:686-741) for one prompt per GPU."""

    def __init__(self, cfg: FluxConfig = FluxConfig(), device="cuda", seed: int = 0,
                 num_double: int | None = None, num_single: int | None = None):
        self.cfg, self.device = cfg, torch.device(device)
        h = cfg.hidden_size
        pd = cfg.patch_size ** 2 * cfg.in_channels
        # patch / text / time projections are Q8_0 linears too (patch_dim 64, time_dim 256
        # and text_dim 4096 all satisfy K % 64 == 0)
        ws = cfg.weight_scale
        self.img_embed = _q8_linear(seed + 1, h, pd, device, scale_range=ws)
        self.txt_embed = _q8_linear(seed + 2, h, cfg.text_dim, device, scale_range=ws)
        self.t1 = _q8_linear(seed + 3, h, cfg.time_dim, device, scale_range=ws)
        self.t2 = _q8_linear(seed + 4, h, h, device, scale_range=ws)
        self.g1 = _q8_linear(seed + 5, h, cfg.guidance_dim, device, scale_range=ws)
        self.g2 = _q8_linear(seed + 6, h, h, device, scale_range=ws)
        nd = cfg.num_double_blocks if num_double is None else num_double
        ns = cfg.num_single_blocks if num_single is None else num_single
        self.double = [FluxDoubleBlockB200(seed + 100 + 50 * i, cfg, device) for i in range(nd)]
        self.single = [FluxSingleBlockB200(seed + 5000 + 50 * i, cfg, device) for i in range(ns)]
        self.final_mod = _q8_linear(seed + 7, 2 * h, h, device, scale_range=ws)
        self.final_proj = _q8_linear(seed + 8, pd, h, device, scale_range=ws)
        cos, sin = rope_tables(cfg.head_dim, cfg.max_seq_len)
        self.cos = torch.from_numpy(cos).to(self.device, torch.bfloat16)
        self.sin = torch.from_numpy(sin).to(self.device, torch.bfloat16)
        # the GEMM-epilogue RoPE reads f32 (cos, sin) pairs of the unrounded angles
        self.cos._sp_rope_pairs = rope_pair_table(torch.from_numpy(cos), torch.from_numpy(sin)).to(self.device)
        self.tfreq = torch.from_numpy(flux_timestep_freqs(cfg.time_dim)).to(self.device)
        self.act_dtype = torch.bfloat16  # activations entering the GEMMs
        self.gfreq = torch.from_numpy(flux_timestep_freqs(cfg.guidance_dim)).to(self.device)

    def _temb(self, t: float, freqs, l1, l2):
        a = freqs * t
        e = torch.cat([torch.sin(a), torch.cos(a)])[None].to(self.act_dtype)
        return l2(F.silu(l1(e)))

    def forward(self, latents: torch.Tensor, timestep: float, txt_embeds: torch.Tensor,
                guidance: float | None = None) -> torch.Tensor:
        cfg = self.cfg
        B, C, Hh, Ww = latents.shape
        ps = cfg.patch_size
        ph, pw = Hh // ps, Ww // ps
        # PatchEmbed (dit.rs:299-315): reshape, swap_dims(2,4), swap_dims(3,5), reshape
        x = latents.to(self.act_dtype).reshape(B, C, ph, ps, pw, ps).permute(0, 1, 4, 5, 2, 3)
        img = self.img_embed(x.reshape(B, ph * pw, C * ps * ps))
        txt = self.txt_embed(txt_embeds.to(self.act_dtype))
        cond = self._temb(timestep, self.tfreq, self.t1, self.t2)
        if guidance is not None:
            cond = cond + self._temb(guidance, self.gfreq, self.g1, self.g2)
        for blk in self.double:
            img, txt = blk.forward(img, txt, cond, self.cos, self.sin)
        x = torch.cat([img, txt], dim=1)
        for blk in self.single:
            x = blk.forward(x, cond, self.cos, self.sin)
        x = x[:, : ph * pw]
        m = self.final_mod(cond).view(B, 1, 2 * cfg.hidden_size)
        shift, scale = m[..., : cfg.hidden_size], m[..., cfg.hidden_size:]
        out = self.final_proj(_ln(x, scale, shift))
        # unpatchify (dit.rs:326-345): reshape [B, ph, pw, C, ps, ps], swap_dims(2, 4),
        # swap_dims(3, 5), reshape [B, C, H, W] -- the element order of the two swaps
        out = out.reshape(B, ph, pw, C, ps, ps).permute(0, 1, 4, 5, 2, 3)
        return out.reshape(B, C, Hh, Ww)

    __call__ = forward


def flux_step_flops(cfg: FluxConfig = FluxConfig(), img_tokens=4096, txt_tokens=512,
                    num_double=None, num_single=None) -> float:
    """Algorithmic FLOPs of the blocks of one Flux step (2 per MAC; linears + attention)."""
    h, i, H, D = cfg.hidden_size, cfg.intermediate, cfg.num_heads, cfg.head_dim
    nd = cfg.num_double_blocks if num_double is None else num_double
    ns = cfg.num_single_blocks if num_single is None else num_single
    S = img_tokens + txt_tokens
    lin = lambda m, n, k: 2.0 * m * n * k  # noqa: E731
    dbl = 0.0
    for s_self, s_other in ((img_tokens, txt_tokens), (txt_tokens, img_tokens)):
        dbl += lin(s_self, 3 * h, h) + lin(s_other, 2 * h, h) + lin(s_self, h, h)
        dbl += lin(s_self, 2 * i, h) + lin(s_self, h, i)
        dbl += 4.0 * H * s_self * S * D
    dbl += lin(1, 6 * h, h)
    sgl = lin(S, 3 * h, h) + lin(S, h, h) + lin(S, 2 * i, h) + lin(S, h, i) + 4.0 * H * S * S * D
    sgl += lin(1, 3 * h, h)
    return nd * dbl + ns * sgl


__all__ = ["FluxConfig", "FluxB200", "FluxDoubleBlockB200", "FluxSingleBlockB200",
           "flux_step_flops", "rope_tables", "apply_rope", "flux_timestep_freqs"]
