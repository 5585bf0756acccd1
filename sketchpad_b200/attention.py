"""Flash attention: host mirror of sketchpad_cubecl::attention and sketchpad_core::attention.

Reference interface (rhi-zone/sketchpad):
  crates/sketchpad-cubecl/src/attention.rs:40-68   FlashAttentionOptions { out_dtype, causal }
  crates/sketchpad-cubecl/src/attention.rs:97       flash_attention(q, k, v, options)
  crates/sketchpad-cubecl/src/attention.rs:119      flash_attention_masked(q, k, v, mask, options)
  crates/sketchpad-core/src/attention.rs:4-27       qkv_attention(q, k, v, mask)
  crates/sketchpad-core/src/attention.rs:33-42      causal_mask(seq_len)
Tensors are [batch, heads, seq, head_dim] CUDA tensors with any strides whose last stride is 1
(e.g. the `reshape(..).swap_dims(1, 2)` views of the UNet/DiT callers).  The kernel computes in
bf16/f16 with an f32 accumulator; f32 inputs are rounded to bf16 on the device first.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, replace
from typing import Optional

import torch

from . import _lib
from ._torch import dtype_code, ptr, require_cuda, stream_ptr, strides4


class AttentionSetupError(RuntimeError):
    """Raised where the reference returns Err(AttentionSetupError) (attention.rs:97-104)."""


@dataclass(frozen=True)
class FlashAttentionOptions:
    """attention.rs:40-68.  out_dtype None = the query dtype."""

    out_dtype: Optional[torch.dtype] = None
    causal: bool = False

    @staticmethod
    def new_causal() -> "FlashAttentionOptions":
        """FlashAttentionOptions::causal()."""
        return FlashAttentionOptions(None, True)

    def with_dtype(self, dtype: torch.dtype) -> "FlashAttentionOptions":
        return replace(self, out_dtype=dtype)

    def with_causal(self, causal: bool) -> "FlashAttentionOptions":
        return replace(self, causal=causal)


def _prep(t: torch.Tensor, compute: torch.dtype) -> torch.Tensor:
    if t.dtype != compute:
        t = t.to(compute)
    if t.stride(-1) != 1 or any((s * t.element_size()) % 16 for s in t.stride()[:-1]) \
            or t.data_ptr() % 16:
        t = t.contiguous()
    return t


def _flash(query, key, value, mask, options: FlashAttentionOptions, scale, out):
    if query.dim() != 4 or key.dim() != 4 or value.dim() != 4:
        raise AttentionSetupError("query, key and value must be [batch, heads, seq, dim]")
    dev = require_cuda(query, key, value, mask, out)
    B, H, Sq, D = query.shape
    Bk, Hk, Skv, Dk = key.shape
    Bv, Hv, Skv2, Dv = value.shape
    if (Bk, Hk, Dk) != (B, H, D) or (Bv, Hv, Skv2) != (B, H, Skv):
        raise AttentionSetupError(
            f"shape mismatch q{tuple(query.shape)} k{tuple(key.shape)} v{tuple(value.shape)}")
    compute = query.dtype if query.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16
    q, k, v = (_prep(t, compute) for t in (query, key, value))
    # the output dtype: the options', else a given out's (bf16 / f16 / f32), else the query's
    out_dtype = options.out_dtype or (out.dtype if out is not None else query.dtype)
    if out is None:
        out = torch.empty((B, H, Sq, Dv), dtype=out_dtype, device=dev)
    elif out.shape != (B, H, Sq, Dv) or out.dtype != out_dtype:
        raise AttentionSetupError("out has the wrong shape or dtype")
    m = None
    mstride = 0
    if mask is not None:
        if mask.dim() != 2 or mask.shape != (Sq, Skv):
            raise AttentionSetupError(f"mask must be [seq_q, seq_k] = [{Sq}, {Skv}]")
        m = mask.to(torch.float32)
        if m.stride(-1) != 1:
            m = m.contiguous()
        mstride = m.stride(0)
    try:
        _lib.call("sp_flash_attn_fwd", ptr(q), ptr(k), ptr(v), ptr(m), mstride, ptr(out), B, H, Sq,
                  Skv, D, Dv, strides4(q), strides4(k), strides4(v), strides4(out),
                  dtype_code(compute), dtype_code(out_dtype), 1 if options.causal else 0,
                  float(scale) if scale else 0.0, stream_ptr(dev))
    except _lib.SketchpadError as e:
        raise AttentionSetupError(str(e)) from e
    return out


def flash_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                    options: FlashAttentionOptions = FlashAttentionOptions(), *,
                    scale: Optional[float] = None, out: Optional[torch.Tensor] = None):
    """softmax(Q K^T / sqrt(d) [causal]) V -> [batch, heads, seq_q, val_dim] (attention.rs:97)."""
    return _flash(query, key, value, None, options, scale, out)


def flash_attention_masked(query, key, value, mask: torch.Tensor,
                           options: FlashAttentionOptions = FlashAttentionOptions(), *,
                           scale: Optional[float] = None, out: Optional[torch.Tensor] = None):
    """Same with an additive [seq_q, seq_k] mask (attention.rs:119)."""
    return _flash(query, key, value, mask, options, scale, out)


def qkv_attention(q, k, v, mask: Optional[torch.Tensor] = None):
    """sketchpad_core::attention::qkv_attention: softmax((q d^-1/4)(k d^-1/4)^T + mask) v.

    (q s)(k s)^T = q k^T s^2 with s^2 = d^-1/2, i.e. the flash kernel's default scale."""
    d = q.shape[-1]
    opts = FlashAttentionOptions()
    scale = d ** -0.5
    if mask is None:
        return flash_attention(q, k, v, opts, scale=scale)
    return flash_attention_masked(q, k, v, mask, opts, scale=scale)


def causal_mask(seq_len: int, device) -> torch.Tensor:
    """sketchpad_core::attention::causal_mask: -inf above the diagonal."""
    m = torch.full((seq_len, seq_len), float("-inf"), device=device)
    return torch.triu(m, diagonal=1)


def attention_flops(B, H, Sq, Skv, D, Dv=None) -> float:
    """Algorithmic FLOPs (2 for QK^T, 2 for PV per MAC, unpadded head dims)."""
    Dv = D if Dv is None else Dv
    return 2.0 * B * H * Sq * Skv * (D + Dv)


__all__ = ["AttentionSetupError", "FlashAttentionOptions", "flash_attention",
           "flash_attention_masked", "qkv_attention", "causal_mask", "attention_flops"]

_ = math  # imported for users computing scales
