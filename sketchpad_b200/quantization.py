"""FP8 (e4m3) weights: host mirror of the FP8 API of crates/sketchpad-core/src/quantization.rs.

  :311-368  Fp8Format (E4M3 / E5M2 constants)
  :372-419  Fp8Config { format, per_channel, scale }
  :422-447  Fp8Tensor { data, scale, format, shape } + dequantize()
  :495-577  quantize_fp8(tensor, config)
  :580-615  Fp8Linear { from_weight, forward, memory_ratio }
The reference simulates FP8 by keeping rounded values in f32; here `data` holds real e4m3
bytes on the GPU (uint8 tensor) and Fp8Linear.forward decodes them inside the GEMM
mainloop with the per-channel scale applied in the epilogue.  Only E4M3 runs on the GPU.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass, replace
from typing import Optional

import torch

from . import _lib
from ._torch import dtype_code, ptr, require_cuda, stream_ptr


class Fp8Format(enum.Enum):
    E4M3 = "e4m3"
    E5M2 = "e5m2"

    def exponent_bits(self) -> int:
        return 4 if self is Fp8Format.E4M3 else 5

    def mantissa_bits(self) -> int:
        return 3 if self is Fp8Format.E4M3 else 2

    def bias(self) -> int:
        return 7 if self is Fp8Format.E4M3 else 15

    def max_value(self) -> float:
        return 448.0 if self is Fp8Format.E4M3 else 57344.0

    def min_normal(self) -> float:
        return 2.0 ** -6 if self is Fp8Format.E4M3 else 2.0 ** -14

    def min_subnormal(self) -> float:
        return 2.0 ** -9 if self is Fp8Format.E4M3 else 2.0 ** -16


@dataclass(frozen=True)
class Fp8Config:
    format: Fp8Format = Fp8Format.E4M3
    per_channel: bool = False
    scale: Optional[float] = None

    @staticmethod
    def e4m3() -> "Fp8Config":
        return Fp8Config(Fp8Format.E4M3)

    @staticmethod
    def e5m2() -> "Fp8Config":
        return Fp8Config(Fp8Format.E5M2)

    def with_per_channel(self, per_channel: bool) -> "Fp8Config":
        return replace(self, per_channel=per_channel)

    def with_scale(self, scale: float) -> "Fp8Config":
        return replace(self, scale=scale)


@dataclass
class Fp8Tensor:
    data: torch.Tensor   # uint8 e4m3 bytes [rows, cols]
    scale: torch.Tensor  # float32 [rows] (per channel) or [1]
    format: Fp8Format
    shape: tuple

    def dequantize(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """Fp8Tensor::dequantize (quantization.rs:435-447): data * scale[row]."""
        dev = require_cuda(self.data, self.scale)
        rows, cols = self.shape
        out = torch.empty((rows, cols), dtype=dtype, device=dev)
        _lib.call("sp_fp8_dequant", ptr(self.data), ptr(self.scale), self.scale.numel(), rows,
                  cols, ptr(out), dtype_code(dtype), stream_ptr(dev))
        return out


def quantize_fp8(tensor: torch.Tensor, config: Fp8Config = Fp8Config()) -> Fp8Tensor:
    """quantize_fp8 (quantization.rs:495-577) on the GPU, E4M3 only."""
    if config.format is not Fp8Format.E4M3:
        raise ValueError("only E4M3 has a GPU encoding")
    dev = require_cuda(tensor)
    w = tensor.to(torch.float32).contiguous()
    rows, cols = w.shape
    data = torch.empty((rows, cols), dtype=torch.uint8, device=dev)
    if config.per_channel:
        scale = torch.empty(rows, dtype=torch.float32, device=dev)
        mode = 1
    elif config.scale is not None:
        scale = torch.full((1,), float(config.scale), dtype=torch.float32, device=dev)
        mode = 2
    else:
        scale = torch.empty(1, dtype=torch.float32, device=dev)
        mode = 0
    _lib.call("sp_fp8_quantize", ptr(w), rows, cols, mode, ptr(data), ptr(scale), stream_ptr(dev))
    return Fp8Tensor(data, scale, config.format, (rows, cols))


class Fp8Linear:
    """quantization.rs:580-615: y = x @ dequant(W)^T + b with W stored as e4m3 + scales."""

    def __init__(self, weight: Fp8Tensor, bias: Optional[torch.Tensor] = None):
        self.weight, self.bias = weight, bias

    @classmethod
    def from_weight(cls, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
                    config: Fp8Config = Fp8Config()):
        return cls(quantize_fp8(weight, config), bias)

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None,
                gate: Optional[torch.Tensor] = None,
                residual: Optional[torch.Tensor] = None, rope=None,
                glu: Optional[int] = None, out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """x @ dequant(W)^T + b; with gate / residual: residual + gate * (x @ W^T + b); with
        `rope` (a RopeEpilogue) the rotary embedding of its columns, and `out` may be a
        column slice of a wider buffer."""
        dev = require_cuda(x, self.weight.data, gate, residual,
                           None if rope is None else rope.table)
        N, K = self.weight.shape
        lead = x.shape[:-1]
        xx = x.reshape(-1, K)
        if xx.dtype != torch.bfloat16:
            xx = xx.to(torch.bfloat16)
        xx = xx.contiguous()
        M = xx.shape[0]
        b = self.bias
        if b is not None and b.dtype != torch.bfloat16:
            b = b.to(torch.bfloat16)
        if glu is not None:  # rows interleaved (first-half j, second-half j): y [.., N/2]
            if gate is not None or residual is not None or rope is not None:
                raise ValueError("the GLU epilogue takes no gate, residual or rope")
            y = out if out is not None else torch.empty((M, N // 2), dtype=torch.bfloat16, device=dev)
            if y.dtype != torch.bfloat16 or not y.is_contiguous() or y.numel() != M * (N // 2):
                raise ValueError("out must be a contiguous bf16 tensor of [..., N / 2]")
            _lib.call("sp_fp8_linear_glu", ptr(xx), ptr(self.weight.data), ptr(self.weight.scale),
                      self.weight.scale.numel(), ptr(b), ptr(y), M, N, K, int(glu), _lib.SP_BF16,
                      stream_ptr(dev))
            return y.reshape(*lead, N // 2)
        f16_out = out_dtype == torch.float16 or (out is not None and out.dtype == torch.float16)
        if rope is not None or f16_out or (out is not None and not out.is_contiguous()):
            from .quantized_matmul import _NO_ROPE, _output_rows
            if gate is not None or residual is not None:
                raise ValueError("the rope / strided-output epilogue takes no gate or residual")
            y, ldy = _output_rows(out, M, N, dev, torch.float16 if f16_out else torch.bfloat16)
            r = rope.args() if rope is not None else _NO_ROPE
            _lib.call("sp_fp8_linear_rope", ptr(xx), ptr(self.weight.data),
                      ptr(self.weight.scale), self.weight.scale.numel(), ptr(b), ptr(y), ldy, M,
                      N, K, *r, _lib.SP_F16 if f16_out else _lib.SP_BF16, stream_ptr(dev))
            return y if out is not None else y.reshape(*lead, N)
        y = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        if gate is None and residual is None:
            _lib.call("sp_fp8_linear", ptr(xx), ptr(self.weight.data), ptr(self.weight.scale),
                      self.weight.scale.numel(), ptr(b), ptr(y), M, N, K, _lib.SP_BF16,
                      stream_ptr(dev))
        else:
            from .quantized_matmul import _epilogue_operands
            g, r = _epilogue_operands(gate, residual, M, N)
            _lib.call("sp_fp8_linear_gated", ptr(xx), ptr(self.weight.data),
                      ptr(self.weight.scale), self.weight.scale.numel(), ptr(b), ptr(g), ptr(r),
                      ptr(y), M, N, K, _lib.SP_BF16, stream_ptr(dev))
        y = y.reshape(*lead, N)
        return y if x.dtype == torch.bfloat16 else y.to(x.dtype)

    __call__ = forward

    def memory_ratio(self) -> float:
        return 8.0 / 32.0


def make_fp8_synthetic(out_features: int, in_features: int, device="cuda", seed: int = 0):
    """BASELINE config 5's weights: random e4m3 bytes (NaN codes excluded) and per-output
    channel f32 scales."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    data = torch.randint(0, 256, (out_features, in_features), generator=g, dtype=torch.int32)
    data = torch.where((data & 0x7F) == 0x7F, data - 1, data).to(torch.uint8)
    scale = (torch.rand(out_features, generator=g) * 0.004 + 0.0005).to(torch.float32)
    return Fp8Tensor(data.to(device), scale.to(device), Fp8Format.E4M3, (out_features, in_features))


__all__ = ["Fp8Format", "Fp8Config", "Fp8Tensor", "quantize_fp8", "Fp8Linear",
           "make_fp8_synthetic"]
