"""Gated-linear-unit gates of the feed-forwards, one pass over the stacked hidden tensor.

Reference semantics (rhi-zone/sketchpad):
  GEGLU   crates/sketchpad-unet/src/blocks.rs:446-458   value * gelu(gate), value = first half
  SwiGLU  crates/sketchpad-core/src/glu.rs:91-96         silu(gate) * up, gate = first half
          (the Flux blocks' SwiGluFfn; WanExpert::forward, crates/sketchpad-dit/src/wan.rs:330-337)
The GEMM producing the hidden tensor stacks both halves (one [M, 2F] output), so the gate
reads it once and writes [M, F].
"""
from __future__ import annotations

import torch

from . import _lib
from ._torch import dtype_code, ptr, require_cuda, stream_ptr

SP_GLU_GEGLU = 0
SP_GLU_SWIGLU = 1


def _gate(hidden: torch.Tensor, kind: int, out=None) -> torch.Tensor:
    dev = require_cuda(hidden, out)
    two_f = hidden.shape[-1]
    if two_f % 2:
        raise ValueError("the last dimension must hold two equal halves")
    F = two_f // 2
    x = hidden.reshape(-1, two_f)
    if x.stride(-1) != 1:
        x = x.contiguous()
    rows = x.shape[0]
    y = out if out is not None else torch.empty(hidden.shape[:-1] + (F,), dtype=hidden.dtype,
                                                device=dev)
    _lib.call("sp_glu_gate", ptr(x), ptr(y), rows, F, x.stride(0), F, kind,
              dtype_code(hidden.dtype), stream_ptr(dev))
    return y


def geglu(hidden: torch.Tensor, out=None) -> torch.Tensor:
    """hidden[..., :F] * gelu(hidden[..., F:]) (erf GELU)."""
    return _gate(hidden, SP_GLU_GEGLU, out)


def swiglu(hidden: torch.Tensor, out=None) -> torch.Tensor:
    """silu(hidden[..., :F]) * hidden[..., F:]."""
    return _gate(hidden, SP_GLU_SWIGLU, out)


__all__ = ["geglu", "swiglu", "SP_GLU_GEGLU", "SP_GLU_SWIGLU"]
