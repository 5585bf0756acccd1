"""Fused GroupNorm(+SiLU): host mirror of sketchpad_cubecl::groupnorm_silu.

Reference interface (rhi-zone/sketchpad):
  crates/sketchpad-cubecl/src/groupnorm_silu.rs:22-46   GroupNormSiLuOptions { num_groups, eps }
  crates/sketchpad-cubecl/src/groupnorm_silu.rs:232     groupnorm_silu(input, weight, bias, options)
  crates/sketchpad-cubecl/src/groupnorm_silu.rs:323     groupnorm(input, weight, bias, options)
  crates/sketchpad-cubecl/src/groupnorm_silu.rs:436-485 GroupNormSiLuLayer
Semantics follow the CPU GroupNorm (crates/sketchpad-core/src/groupnorm.rs:62-102): clamp
+-65000, f32 statistics with the biased variance, clamp after the affine.  The reference
panics when channels % num_groups != 0; this raises ValueError.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._torch import dtype_code, ptr, require_cuda, stream_ptr


@dataclass(frozen=True)
class GroupNormSiLuOptions:
    num_groups: int = 32
    eps: float = 1e-5

    @staticmethod
    def with_groups(num_groups: int) -> "GroupNormSiLuOptions":
        return GroupNormSiLuOptions(num_groups, 1e-5)


def _run(input: torch.Tensor, weight, bias, options: GroupNormSiLuOptions, act: int,
         out=None, add=None) -> torch.Tensor:
    if input.dim() != 4:
        raise ValueError("input must be [batch, channels, height, width]")
    dev = require_cuda(input, weight, bias, out)
    B, C, H, W = input.shape
    G = options.num_groups
    if C % G != 0:
        raise ValueError(f"channels ({C}) must be divisible by num_groups ({G})")
    if weight.numel() != C or bias.numel() != C:
        raise ValueError("weight/bias length must equal channels")
    dt = input.dtype
    w = weight if weight.dtype == dt else weight.to(dt)
    b = bias if bias.dtype == dt else bias.to(dt)
    w, b = w.contiguous(), b.contiguous()
    channels_last = (not input.is_contiguous()) and input.is_contiguous(
        memory_format=torch.channels_last)
    if out is None:
        fmt = torch.channels_last if channels_last else torch.contiguous_format
        out = torch.empty((B, C, H, W), dtype=dt, device=dev, memory_format=fmt)
    code = dtype_code(dt)
    strides = _lib.i64_array(input.stride())
    ws_bytes = _lib.load().sp_groupnorm_act_workspace_size(B, C, H, W, strides, G, code)
    if ws_bytes == 0 and (input.data_ptr() % 16 or out.data_ptr() % 16):
        # misaligned views take the two-pass path as well
        ws_bytes = _lib.load().sp_groupnorm_act_workspace_size(B, C, H, W, _lib.i64_array(
            (1, 1, 1, 1)), G, code) or 4
        ws_bytes = max(ws_bytes, 12 * B * G * ((C // G * H * W + 16383) // 16384))
    ws = None
    if ws_bytes:
        ws = torch.empty((ws_bytes + 3) // 4, dtype=torch.float32, device=dev)
    nws = 0 if ws is None else ws.numel() * 4
    if add is not None:
        if tuple(add.shape) != (B, C):
            raise ValueError("add must be [batch, channels]")
        a = (add if add.dtype == dt else add.to(dt)).contiguous()
        _lib.call("sp_groupnorm_add_act", ptr(input), ptr(a), ptr(w), ptr(b), ptr(out), B, C, H,
                  W, strides, G, float(options.eps), act, code, ptr(ws), nws, stream_ptr(dev))
        return out
    _lib.call("sp_groupnorm_act", ptr(input), ptr(w), ptr(b), ptr(out), B, C, H, W, strides, G,
              float(options.eps), act, code, ptr(ws), nws, stream_ptr(dev))
    return out


def groupnorm_silu(input, weight, bias, options: GroupNormSiLuOptions = GroupNormSiLuOptions(),
                   out=None, add=None):
    """silu(groupnorm(x)) in one pass over HBM (groupnorm_silu.rs:232).

    add: optional [batch, channels] tensor; normalises x + add[:, :, None, None] without
    storing the sum (ResBlock's time-embedding add, crates/sketchpad-unet/src/cubecl.rs:115-124).
    Channels-last x only."""
    return _run(input, weight, bias, options, _lib.SP_ACT_SILU, out, add)


def groupnorm(input, weight, bias, options: GroupNormSiLuOptions = GroupNormSiLuOptions(),
              out=None):
    """GroupNorm without the activation (groupnorm_silu.rs:323)."""
    return _run(input, weight, bias, options, _lib.SP_ACT_NONE, out)


class GroupNormSiLuLayer:
    """groupnorm_silu.rs:436-485: fused GroupNorm + SiLU with stored weight/bias."""

    def __init__(self, num_groups: int, weight, bias, eps: float = 1e-5):
        self.num_groups, self.weight, self.bias, self.eps = num_groups, weight, bias, eps

    @classmethod
    def from_tensors(cls, num_groups, weight, bias):
        return cls(num_groups, weight, bias, 1e-5)

    @classmethod
    def from_tensors_with_eps(cls, num_groups, weight, bias, eps):
        return cls(num_groups, weight, bias, eps)

    def forward(self, input):
        return groupnorm_silu(input, self.weight, self.bias,
                              GroupNormSiLuOptions(self.num_groups, self.eps))

    __call__ = forward


def groupnorm_bytes(B, C, H, W, elem_size: int) -> int:
    """Algorithmic HBM bytes: one read and one write of x, plus gamma and beta."""
    return B * C * H * W * 2 * elem_size + 2 * C * elem_size


__all__ = ["GroupNormSiLuOptions", "groupnorm_silu", "groupnorm", "GroupNormSiLuLayer",
           "groupnorm_bytes"]
