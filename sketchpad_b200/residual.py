"""Convolution bias + residual add in one pass (ResBlock::forward,
crates/sketchpad-unet/src/blocks.rs:123-150: conv2(h) + skip(x)).

The UNet harness runs its ResBlock convolutions without bias and adds the biases here
(conv2's and the skip convolution's, pre-summed) together with the residual."""
from __future__ import annotations

import torch

from . import _lib
from ._torch import dtype_code, ptr, require_cuda, stream_ptr


def _rows_c(t: torch.Tensor):
    """[B, C, H, W] channels-last (or [.., C] contiguous) -> (rows, C)."""
    if t.dim() == 4:
        if not t.is_contiguous(memory_format=torch.channels_last):
            raise ValueError("expected a channels-last [B, C, H, W] tensor")
        B, C, H, W = t.shape
        return B * H * W, C
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.numel() // t.shape[-1], t.shape[-1]


def add_bias_residual(y: torch.Tensor, bias: torch.Tensor, residual=None, out=None) -> torch.Tensor:
    """y + bias[channel] (+ residual), same layout as y."""
    dev = require_cuda(y, bias, residual, out)
    rows, C = _rows_c(y)
    if residual is not None and (residual.shape != y.shape or residual.stride() != y.stride()):
        raise ValueError("residual must match y in shape and layout")
    b = (bias if bias.dtype == y.dtype else bias.to(y.dtype)).contiguous()
    if out is None:
        out = torch.empty_like(y)
    _lib.call("sp_add_bias_residual", ptr(y), ptr(residual), ptr(b), ptr(out), rows, C,
              dtype_code(y.dtype), stream_ptr(dev))
    return out


__all__ = ["add_bias_residual"]
