"""LayerNorm with the reference's unbiased variance (crates/sketchpad-core/src/layernorm.rs:63-73).

burn's `var` divides by n - 1, so this is NOT torch.nn.LayerNorm; the UNet and DiT blocks of
the reference normalise this way and the step harness needs the same numbers.
"""
from __future__ import annotations

import torch

from . import _lib
from ._torch import dtype_code, ptr, require_cuda, stream_ptr


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5,
               unbiased: bool = True, out=None, add=None) -> torch.Tensor:
    """LayerNorm over the last dim; with `add` ([n]), of x + add (rounded like an add)."""
    dev = require_cuda(x, weight, bias, out, add)
    n = x.shape[-1]
    xx = x.contiguous()
    dt = xx.dtype
    w = (weight if weight.dtype == dt else weight.to(dt)).contiguous()
    b = (bias if bias.dtype == dt else bias.to(dt)).contiguous()
    y = out if out is not None else torch.empty_like(xx)
    if add is not None:
        a = (add if add.dtype == dt else add.to(dt)).contiguous()
        _lib.call("sp_layernorm_add", ptr(xx), ptr(a), ptr(w), ptr(b), ptr(y), xx.numel() // n,
                  n, float(eps), 1 if unbiased else 0, dtype_code(dt), stream_ptr(dev))
        return y
    _lib.call("sp_layernorm", ptr(xx), ptr(w), ptr(b), ptr(y), xx.numel() // n, n, float(eps),
              1 if unbiased else 0, dtype_code(dt), stream_ptr(dev))
    return y


def layer_norm_modulate(x: torch.Tensor, scale: torch.Tensor | None = None,
                        shift: torch.Tensor | None = None, eps: float = 1e-5,
                        unbiased: bool = True, out=None) -> torch.Tensor:
    """LN(x) * (1 + scale) + shift over x [b, s, n] with LN = LayerNorm::new (gamma 1, beta 0)
    and scale / shift of shape [b, 1, n] (any strides whose last dim is contiguous: slices of
    the modulation output), one pass (crates/sketchpad-dit/src/flux.rs:479-481)."""
    dev = require_cuda(x, scale, shift, out)
    xx = x.contiguous()
    b, n = xx.shape[0], xx.shape[-1]
    rows = xx.numel() // n
    stride = None
    ops = []
    for v in (scale, shift):
        if v is None:
            ops.append(None)
            continue
        if v.dtype != xx.dtype:
            raise ValueError("scale / shift must have x's dtype")
        v2 = v.reshape(v.shape[0], -1) if v.dim() > 1 else v.reshape(1, -1)
        if v2.shape != (b, n) and not (v2.shape == (1, n) and b == 1):
            raise ValueError(f"scale / shift must hold one [{n}] vector per batch entry")
        if v2.stride(-1) != 1:
            raise ValueError("scale / shift rows must be contiguous")
        s = v2.stride(0) if b > 1 else 0
        if stride is not None and s != stride:
            raise ValueError("scale and shift must share the batch stride")
        stride = s
        ops.append(v2)
    y = out if out is not None else torch.empty_like(xx)
    _lib.call("sp_layernorm_modulate", ptr(xx), ptr(ops[0]), ptr(ops[1]), ptr(y), rows, n,
              rows // b, stride or 0, float(eps), 1 if unbiased else 0, dtype_code(xx.dtype),
              stream_ptr(dev))
    return y


class LayerNorm:
    """sketchpad_core::layernorm::LayerNorm { weight, bias, eps }."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5):
        self.weight, self.bias, self.eps = weight, bias, eps

    @classmethod
    def new(cls, size: int, device="cuda", dtype=torch.bfloat16):
        return cls(torch.ones(size, device=device, dtype=dtype),
                   torch.zeros(size, device=device, dtype=dtype))

    def forward(self, x):
        return layer_norm(x, self.weight, self.bias, self.eps, True)

    __call__ = forward


__all__ = ["LayerNorm", "layer_norm", "layer_norm_modulate"]
