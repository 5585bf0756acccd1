"""Bf16Linear: y = x W^T + b with plain bf16 weights on the library's tcgen05 GEMM
(sp_bf16_linear* in include/sketchpad_b200.h), with the same epilogues as the quantized
linears: bias, in-place residual accumulation (residual + gate * (x W^T + b)) and the
GEGLU / SwiGLU gate over row-interleaved weights.

UNetB200(gemm="sp") runs every projection and feed-forward GEMM of the SD1.x step on it --
the burn Linear layers of crates/sketchpad-unet/src/blocks.rs:213-231, :292-305, :370-410,
:446-458 (the step's default stays cuBLAS: the 256 x 256 tiles underfill the SMs on those
small-K products).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from ._torch import ptr, require_cuda, stream_ptr
from .quantized_matmul import _epilogue_operands, interleave_rows


class Bf16Linear:
    """weight [out_features, in_features] bf16 (torch / GGUF row order; burn stores [in, out]
    and computes x @ W, the same product), optional bias [out_features]."""

    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                 dtype: torch.dtype = torch.bfloat16):
        """dtype: the stored weight type; the GPU kernel takes bf16 (another dtype only serves
        host-side stand-ins of the kernel, e.g. wiring tests)."""
        if weight.dim() != 2:
            raise ValueError("weight must be [out_features, in_features]")
        self.weight = weight.to(dtype).contiguous()
        self.out_features, self.in_features = self.weight.shape
        if self.in_features % 64 or self.out_features % 16:
            raise ValueError("in_features must be a multiple of 64 and out_features of 16")
        self.bias = None if bias is None else bias.reshape(-1).to(self.weight.device,
                                                                  dtype).contiguous()

    @classmethod
    def from_in_out(cls, w_kn: torch.Tensor, bias: Optional[torch.Tensor] = None) -> "Bf16Linear":
        """From burn's [in_features, out_features] layout."""
        return cls(w_kn.t(), bias)

    @classmethod
    def glu(cls, first: "Bf16Linear", second: "Bf16Linear") -> "Bf16Linear":
        """One layer whose rows interleave two halves (first j, second j): its `glu` forward
        gives lo * gelu(hi) / silu(lo) * hi without storing the [M, 2F] product."""
        b = None
        dt = first.weight.dtype
        if first.bias is not None or second.bias is not None:
            z = lambda l: l.bias if l.bias is not None else torch.zeros(  # noqa: E731
                l.out_features, dtype=dt, device=l.weight.device)
            b = interleave_rows(z(first), z(second))
        return cls(interleave_rows(first.weight, second.weight), b, dt)

    def forward(self, input: torch.Tensor, out: Optional[torch.Tensor] = None,
                gate: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
                glu: Optional[int] = None) -> torch.Tensor:
        """[..., in] -> [..., out] (bf16).  With gate / residual: residual + gate * (x W^T + b)
        from the epilogue (residual may be `out`: in-place accumulation); with glu
        (GLU_GEGLU / GLU_SWIGLU): [..., out / 2]."""
        dev = require_cuda(input, self.weight, gate, residual, out)
        lead = input.shape[:-1]
        x = input.reshape(-1, self.in_features)
        x = (x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)).contiguous()
        M, N, K = x.shape[0], self.out_features, self.in_features
        if glu is not None:
            if gate is not None or residual is not None:
                raise ValueError("the GLU epilogue takes no gate or residual")
            y = out if out is not None else torch.empty((M, N // 2), dtype=torch.bfloat16,
                                                        device=dev)
            if y.dtype != torch.bfloat16 or not y.is_contiguous() or y.numel() != M * (N // 2):
                raise ValueError("out must be a contiguous bf16 tensor of [..., out / 2]")
            _lib.call("sp_bf16_linear_glu", ptr(x), ptr(self.weight), ptr(self.bias), ptr(y), M,
                      N, K, int(glu), _lib.SP_BF16, stream_ptr(dev))
            return y.reshape(*lead, N // 2)
        y = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        if y.dtype != torch.bfloat16 or not y.is_contiguous() or y.numel() != M * N:
            raise ValueError("out must be a contiguous bf16 tensor of the output's shape")
        if gate is None and residual is None:
            _lib.call("sp_bf16_linear", ptr(x), ptr(self.weight), ptr(self.bias), ptr(y), M, N,
                      K, _lib.SP_BF16, stream_ptr(dev))
        else:
            g, r = _epilogue_operands(gate, residual, M, N)
            _lib.call("sp_bf16_linear_gated", ptr(x), ptr(self.weight), ptr(self.bias), ptr(g),
                      ptr(r), ptr(y), M, N, K, _lib.SP_BF16, stream_ptr(dev))
        return y.reshape(*lead, N)

    __call__ = forward


__all__ = ["Bf16Linear"]
