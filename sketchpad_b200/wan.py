"""Wan-2.1-14B-shaped video DiT block with FP8 weights on the B200 kernels,
optionally sequence-parallel (Ulysses) across the ranks of a process group.

Follows rhi-zone/sketchpad crates/sketchpad-dit/src/wan.rs:
  :188-221   wan_timestep_freqs / WanTimestepEmbed
  :330-337   WanExpert (SwiGLU, no bias): down(silu(gate(x)) * up(x))
  :351-402   WanAttention (to_qkv -> RoPE(q,k) -> softmax(QK^T/sqrt(d))V -> to_out)
  :418-461   WanCrossAttention (to_q(x), to_kv(context))
  :489-573   WanBlock::forward: 8x modulation; spatial attention over each frame's H*W tokens,
             temporal attention over T frames per position, text cross-attention, MoE FFN
  :576-601   forward_moe: softmax router, dense sum over experts (num_experts = 1 here, so
             the router weight is exactly 1 and the FFN is one SwiGLU expert)
  :613-627   WanFinalLayer, :661-718 patchify / unpatchify, :720-757 Wan::forward
Config 5: hidden 5120, 40 heads x 128, FFN 13824, 40 blocks, latent 16x21x90x160 with patch
1x2x2 -> 21 frames x 45 x 80 = 75,600 tokens, text context 512 x 4096 (projected to hidden).

Every Linear is an Fp8Linear (e4m3 bytes + per-output-channel f32 scale, decode fused into
the GEMM mainloop).  Sequence parallel: each rank holds S/P tokens; around each attention
`ulysses` regroups to all tokens x H/P heads with one all-to-all per tensor.  Spatial and
temporal attention are then computed exactly as on one device; the cross-attention needs
only the rank's own queries and the (replicated) 512-token context.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F

from .attention import flash_attention
from .flux import apply_rope, rope_tables
from .quantized_matmul import GLU_SWIGLU, RopeEpilogue, interleave_rows, rope_pair_table
from .layernorm import layer_norm_modulate
from .quantization import Fp8Format, Fp8Linear, Fp8Tensor
from .ulysses import all_gather_tokens, head_to_seq, rank_of, seq_to_head_qkv, world_size


@dataclass(frozen=True)
class WanConfig:
    in_channels: int = 16
    patch_size: int = 2
    temporal_patch_size: int = 1
    hidden_size: int = 5120
    num_heads: int = 40
    num_blocks: int = 40
    intermediate: int = 13824
    text_dim: int = 4096
    time_embed_dim: int = 256
    max_spatial_len: int = 3600
    max_temporal_len: int = 21
    # dtype of the attention inputs q, k, v written by the projection epilogues: f16 keeps
    # 3 more mantissa bits than bf16, so at full width (logits of order 10) the softmax
    # weights move ~8x less than with bf16 q and k; the DiT's q / k / v stay far inside f16's
    # range.  The residual stream and every other activation stay bf16.
    attn_dtype: torch.dtype = torch.float16

    @property
    def head_dim(self):
        return self.hidden_size // self.num_heads


def wan_timestep_freqs(dim: int) -> np.ndarray:
    """wan.rs:188-196: exp(-ln(10000)/(half-1) * i)."""
    half = dim // 2
    s = np.float32(-math.log(10000.0)) / np.float32(half - 1)
    return np.exp(s * np.arange(half, dtype=np.float32)).astype(np.float32)


def fp8_linear_synthetic(seed: int, n: int, k: int, device, bias: bool) -> Fp8Linear:
    """Random e4m3 weight bytes (finite codes) with per-output-channel scales sized so that
    dequantized weights are ~N(0, 0.02)-like, plus an optional bf16 bias ~ N(0, 0.02)."""
    g = torch.Generator(device=device).manual_seed(seed)
    # draw values in the e4m3 range and encode them on the device: N(0,1) * 64 -> e4m3 bytes
    w = torch.randn((n, k), generator=g, device=device) * 64.0
    from .quantization import quantize_fp8, Fp8Config
    t = quantize_fp8(w, Fp8Config.e4m3().with_scale(1.0))
    scale = torch.full((n,), 0.02 / 64.0, device=device, dtype=torch.float32)
    b = (torch.randn(n, generator=g, device=device) * 0.02).to(torch.bfloat16) if bias else None
    return Fp8Linear(Fp8Tensor(t.data, scale, Fp8Format.E4M3, (n, k)), b)


def _ln(x, scale=None, shift=None):
    # LayerNorm::new(hidden) (gamma 1, beta 0, unbiased variance, layernorm.rs:63-73), with
    # the blocks' `(1 + scale) * x + shift` modulation fused when scale / shift are given
    return layer_norm_modulate(x, scale, shift, 1e-5, True)


def _rope_fusable(x):
    # the GEMM epilogue writes bf16
    return x.dtype == torch.bfloat16


class WanBlockB200:
    def __init__(self, seed: int, cfg: WanConfig, device, group=None,
                 rope_dtype: torch.dtype = torch.bfloat16):
        """group: None (one device), a torch.distributed process group or an NcclComm
        (sequence-parallel over its ranks)."""
        h, i = cfg.hidden_size, cfg.intermediate
        L = lambda s, n, k, b=True: fp8_linear_synthetic(seed + s, n, k, device, b)  # noqa: E731
        self.s_qkv, self.s_out = L(1, 3 * h, h), L(2, h, h)
        self.t_qkv, self.t_out = L(3, 3 * h, h), L(4, h, h)
        self.c_q, self.c_kv, self.c_out = L(5, h, h), L(6, 2 * h, h), L(7, h, h)
        gate, up = L(8, i, h, False), L(9, i, h, False)
        # rows interleaved (gate j, up j): silu(gate) * up in the GEMM epilogue
        self.gate_up = Fp8Linear(Fp8Tensor(interleave_rows(gate.weight.data, up.weight.data),
                                           interleave_rows(gate.weight.scale, up.weight.scale),
                                           Fp8Format.E4M3, (2 * i, h)), None)
        self.down = L(10, h, i, False)
        self.modulation = L(11, 8 * h, h)
        self.cfg, self.group = cfg, group
        self.P = world_size(group) if group is not None else 1
        sc, ss = rope_tables(cfg.head_dim, cfg.max_spatial_len)
        tc, ts = rope_tables(cfg.head_dim, cfg.max_temporal_len)
        f = lambda a: torch.from_numpy(a).to(device, rope_dtype)  # noqa: E731
        self.s_cos, self.s_sin, self.t_cos, self.t_sin = f(sc), f(ss), f(tc), f(ts)
        # f32 (cos, sin) pairs of the unrounded angles for the qkv GEMMs' RoPE epilogue
        pairs = lambda c, s_: rope_pair_table(torch.from_numpy(c), torch.from_numpy(s_)).to(device)  # noqa: E731
        self.s_pairs, self.t_pairs = pairs(sc, ss), pairs(tc, ts)

    # attention over the full token sequence of this rank's head group (Ulysses) -----------
    def _self_attn(self, xn, qkv_lin, out_lin, nt, nhw, temporal, residual, out=None):
        cfg, P = self.cfg, self.P
        b, s_loc, _ = xn.shape
        H, D = cfg.num_heads, cfg.head_dim
        # RoPE in the qkv GEMM's epilogue, by each row's global token index (this rank holds
        # tokens [rank * s_loc, (rank + 1) * s_loc) of every sequence); spatial position =
        # token % (h*w), temporal position = token // (h*w) (frame-major tokens)
        fused = _rope_fusable(xn) and (b == 1 or P == 1)
        if fused:
            off = rank_of(self.group) * s_loc if P > 1 else 0
            rope = (RopeEpilogue(self.t_pairs, 2 * H * D, D, off, nhw, nt) if temporal
                    else RopeEpilogue(self.s_pairs, 2 * H * D, D, off, 1, nhw))
            qkv = qkv_lin(xn, rope=rope, out_dtype=cfg.attn_dtype).view(b, s_loc, 3, H, D)
        else:
            qkv = qkv_lin(xn).view(b, s_loc, 3, H, D)
        if P > 1:
            # one exchange for q, k and v; they stay strided views of the receive buffer
            qkv_h = seq_to_head_qkv(qkv, self.group)
            parts = [qkv_h[:, :, j] for j in range(3)]
            hh = H // P
        else:
            parts = [qkv[:, :, j] for j in range(3)]
            hh = H
        # parts: [b, S, hh, D] over all tokens (frame-major: t, then h*w)
        if not temporal:
            q, k, v = (p.reshape(b * nt, nhw, hh, D).transpose(1, 2) for p in parts)
            cos, sin = self.s_cos, self.s_sin
        else:
            q, k, v = (p.reshape(b, nt, nhw, hh, D).permute(0, 2, 3, 1, 4).reshape(b * nhw, hh, nt, D)
                       for p in parts)
            cos, sin = self.t_cos, self.t_sin
        if not fused:
            q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        # attention writes [b, t, h*w, heads, D] directly (strided output view)
        ob = torch.empty((b, nt, nhw, hh, D), dtype=xn.dtype, device=xn.device)
        if not temporal:
            flash_attention(q, k, v, out=ob.view(b * nt, nhw, hh, D).transpose(1, 2))
        elif b == 1:
            flash_attention(q, k, v, out=ob[0].permute(1, 2, 0, 3))
        else:
            o = flash_attention(q, k, v)
            ob.copy_(o.view(b, nhw, hh, nt, D).permute(0, 3, 1, 2, 4))
        o = ob.view(b, nt * nhw, hh, D)
        if P > 1:
            o = head_to_seq(o, self.group)
        # residual + to_out(o), the add done in the GEMM epilogue
        return out_lin(o.reshape(b, s_loc, H * D), out=out, residual=residual)

    def forward(self, x, cond, context, nt: int, nh: int, nw: int):
        """x: [b, S/P, hidden] (this rank's tokens), cond: [b, hidden], context: [b, 512, hidden]."""
        cfg = self.cfg
        b = x.shape[0]
        m = self.modulation(cond).view(b, 8, 1, cfg.hidden_size)
        nhw = nh * nw
        xn = _ln(x, m[:, 1], m[:, 0])
        # the residual adds run in each branch's last GEMM epilogue: out of place for the
        # first (x belongs to the caller), in place on this block's own tensor afterwards
        x = self._self_attn(xn, self.s_qkv, self.s_out, nt, nhw, False, x.contiguous())
        xn = _ln(x, m[:, 3], m[:, 2])
        x = self._self_attn(xn, self.t_qkv, self.t_out, nt, nhw, True, x, out=x)
        xn = _ln(x, m[:, 5], m[:, 4])
        H, D = cfg.num_heads, cfg.head_dim
        s_loc = x.shape[1]
        adt = cfg.attn_dtype if _rope_fusable(xn) else None
        q = self.c_q(xn, out_dtype=adt).view(b, s_loc, H, D).transpose(1, 2)
        kv = self.c_kv(context, out_dtype=adt).view(b, context.shape[1], 2, H, D)
        o = torch.empty((b, s_loc, H, D), dtype=x.dtype, device=x.device)
        flash_attention(q, kv[:, :, 0].transpose(1, 2), kv[:, :, 1].transpose(1, 2),
                        out=o.transpose(1, 2))
        x = self.c_out(o.view(b, s_loc, H * D), out=x, residual=x)
        xn = _ln(x, m[:, 7], m[:, 6])
        # one expert: softmax over a single router logit is exactly 1 (wan.rs:576-601)
        # silu(gate) * up in gate_up's epilogue; the residual add in down's
        return self.down(self.gate_up(xn, glu=GLU_SWIGLU), out=x, residual=x)


class WanB200:
    """Wan::forward (wan.rs:720-757) for one sample: patchify + video_embed, text_embed,
    the timestep embedding (forward_scalar, wan.rs:213-221), the blocks, the final layer
    (wan.rs:613-627) and unpatchify.  Every Linear is an FP8 Linear.

    With a process group of P ranks the sample is sequence-parallel (Ulysses): every rank
    patchifies the whole latent (a few MB) and embeds only its S/P tokens; the blocks
    exchange heads and tokens around each self-attention; the final layer runs on the local
    tokens and one all-gather of the [S/P, C*ps*ps] outputs (S*64*2 bytes in total) gives
    every rank the whole velocity."""

    def __init__(self, cfg: WanConfig = WanConfig(), device="cuda", seed: int = 0,
                 num_blocks: Optional[int] = None, group=None):
        if cfg.temporal_patch_size != 1:
            raise ValueError("temporal_patch_size must be 1 (wan.rs:668)")
        self.cfg, self.device, self.group = cfg, torch.device(device), group
        self.P = world_size(group) if group is not None else 1
        h = cfg.hidden_size
        pd = cfg.in_channels * cfg.patch_size ** 2
        L = lambda s, n, k: fp8_linear_synthetic(seed + s, n, k, device, True)  # noqa: E731
        self.video_embed, self.text_embed = L(1, h, pd), L(2, h, cfg.text_dim)
        self.t1, self.t2 = L(3, h, cfg.time_embed_dim), L(4, h, h)
        nb = cfg.num_blocks if num_blocks is None else num_blocks
        self.blocks = [WanBlockB200(seed + 100 + 20 * i, cfg, device, group) for i in range(nb)]
        self.final_mod, self.final_proj = L(5, 2 * h, h), L(6, pd, h)
        self.freqs = torch.from_numpy(wan_timestep_freqs(cfg.time_embed_dim)).to(self.device)
        self.act_dtype = torch.bfloat16  # activations entering the GEMMs

    def patchify(self, latents: torch.Tensor) -> torch.Tensor:
        """wan.rs:661-689 before the projection: [B, C, T, H, W] -> [B, T*nh*nw, C*ps*ps]."""
        B, C, T, Hh, Ww = latents.shape
        ps = self.cfg.patch_size
        nh, nw = Hh // ps, Ww // ps
        x = latents.permute(0, 2, 1, 3, 4).reshape(B * T, C, nh, ps, nw, ps)
        return x.permute(0, 2, 4, 1, 3, 5).reshape(B, T * nh * nw, C * ps * ps)

    def unpatchify(self, x: torch.Tensor, nt: int, nh: int, nw: int, C: int) -> torch.Tensor:
        """wan.rs:691-718: [B, T*nh*nw, C*ps*ps] -> [B, C, T, H, W]."""
        B = x.shape[0]
        ps = self.cfg.patch_size
        y = x.reshape(B * nt, nh, nw, C, ps, ps).permute(0, 3, 1, 4, 2, 5)
        return y.reshape(B, nt, C, nh * ps, nw * ps).permute(0, 2, 1, 3, 4).contiguous()

    def time_embedding(self, t: float) -> torch.Tensor:
        a = self.freqs * t
        e = torch.cat([torch.sin(a), torch.cos(a)])[None].to(self.act_dtype)
        return self.t2(F.silu(self.t1(e)))

    def forward(self, latents: torch.Tensor, timestep: float, text_embeds: torch.Tensor) -> torch.Tensor:
        cfg, P = self.cfg, self.P
        B, C, T, Hh, Ww = latents.shape
        ps = cfg.patch_size
        nh, nw = Hh // ps, Ww // ps
        x = self.patchify(latents.to(self.act_dtype))
        S = x.shape[1]
        if P > 1:
            if S % P:
                raise ValueError(f"tokens ({S}) must divide by the sequence-parallel size ({P})")
            r = rank_of(self.group)
            x = x[:, r * (S // P):(r + 1) * (S // P)]
        x = self.video_embed(x.contiguous())
        context = self.text_embed(text_embeds.to(self.act_dtype))
        cond = self.time_embedding(timestep)
        for blk in self.blocks:
            x = blk.forward(x, cond, context, T, nh, nw)
        h = cfg.hidden_size
        m = self.final_mod(cond).view(B, 1, 2 * h)
        out = self.final_proj(_ln(x, m[..., h:], m[..., :h]))
        if P > 1:
            out = all_gather_tokens(out, self.group)
        return self.unpatchify(out, T, nh, nw, C)

    __call__ = forward


def wan_step_flops(cfg: WanConfig = WanConfig(), nt=21, nhw=3600, ctx=512, num_blocks=None) -> float:
    """Algorithmic FLOPs of one Wan::forward: the blocks plus the embeddings and final layer."""
    h = cfg.hidden_size
    nb = cfg.num_blocks if num_blocks is None else num_blocks
    S = nt * nhw
    pd = cfg.in_channels * cfg.patch_size ** 2
    extra = 2.0 * (S * pd * h + ctx * cfg.text_dim * h + cfg.time_embed_dim * h + h * h
                   + 2 * h * h + S * h * pd)
    return nb * wan_block_flops(cfg, nt, nhw, ctx)["total"] + extra


def wan_block_flops(cfg: WanConfig = WanConfig(), nt=21, nhw=3600, ctx=512) -> dict:
    """Algorithmic FLOPs of one WanBlock over the whole (unsharded) sequence."""
    h, i, H, D = cfg.hidden_size, cfg.intermediate, cfg.num_heads, cfg.head_dim
    S = nt * nhw
    lin = 2.0 * S * (3 * h * h * 2 + h * h * 2 + h * h + h * h + 2 * i * h + h * i) + \
        2.0 * ctx * 2 * h * h + 2.0 * 8 * h * h
    att = 4.0 * H * D * (nt * nhw * nhw + nhw * nt * nt + S * ctx)
    return {"linear": lin, "attention": att, "total": lin + att}


__all__ = ["WanConfig", "WanB200", "WanBlockB200", "wan_block_flops", "wan_step_flops",
           "wan_timestep_freqs", "fp8_linear_synthetic"]
