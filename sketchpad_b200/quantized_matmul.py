"""GGUF-quantized linear layers (Q8_0, Q4_K, Q2_K, Q3_K) with the dequantization fused into
the GEMM mainloop.

Host mirror of crates/sketchpad-cubecl/src/quantized_matmul.rs:
  :33    GpuQuantType {Q8_0, Q4K, Q2K, Q3K}
  :376   dequantize_q8_0(packed, out_features, in_features); :410-520 the K-quant dequants
  :655   GpuQuantizedLinear { from_bytes :670, dequantize :705, forward_burn :726, forward :752 }
Weights stay quantized in HBM, repacked losslessly: Q8_0 as planar int8 + f16 block scales;
the K-quants as one 4-bit quant per value + two f32 factors per sub-block (see
include/sketchpad_b200.h).  `dequantize()` in f32 is bit-exact with the CPU decode
(crates/sketchpad-convert/src/gguf.rs:643-656 for Q8_0, :737-871 for the K-quants);
`forward` decodes to bf16 inside the GEMM.
"""
from __future__ import annotations

import ctypes
import enum
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._torch import dtype_code, ptr, require_cuda, stream_ptr


class GpuQuantType(enum.Enum):
    Q8_0 = "q8_0"
    Q4K = "q4_k"
    Q2K = "q2_k"
    Q3K = "q3_k"


# GGML type id, bytes per 256-value super-block, values per factor sub-block
_KQ = {GpuQuantType.Q4K: (12, 144, 32), GpuQuantType.Q2K: (10, 84, 16),
       GpuQuantType.Q3K: (11, 110, 16)}


def repack_kquant_host(data, quant_type: GpuQuantType, out_features: int, in_features: int):
    """GGUF K-quant bytes -> (qpack uint8 [out, in/2], a f32 [in/sub, out], b f32 [in/sub, out])
    on the host (the layout of sp_kquant_repack_host)."""
    fmt, _, sub = _KQ[quant_type]
    buf = np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray) else \
        np.ascontiguousarray(data, dtype=np.uint8)
    qp = np.empty((out_features, in_features // 2), np.uint8)
    a = np.empty((in_features // sub, out_features), np.float32)
    b = np.empty_like(a)
    _lib.call("sp_kquant_repack_host", fmt, buf.ctypes.data_as(ctypes.c_void_p), buf.size,
              out_features, in_features, qp.ctypes.data_as(ctypes.c_void_p),
              a.ctypes.data_as(ctypes.c_void_p), b.ctypes.data_as(ctypes.c_void_p))
    return qp, a, b


def dequantize_kquant(quant_type: GpuQuantType, qpack: torch.Tensor, a: torch.Tensor,
                      b: torch.Tensor, out_features: int, in_features: int,
                      dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """dequantize_q4k / dequantize_q2k / dequantize_q3k (quantized_matmul.rs:410-520) from the
    repacked form; f32 output is bit-exact with the CPU decode."""
    dev = require_cuda(qpack, a, b)
    out = torch.empty((out_features, in_features), dtype=dtype, device=dev)
    _lib.call("sp_kquant_dequant", _KQ[quant_type][0], ptr(qpack), ptr(a), ptr(b), out_features,
              in_features, ptr(out), dtype_code(dtype), stream_ptr(dev))
    return out


def repack_q8_0_host(data: bytes | np.ndarray, out_features: int, in_features: int):
    """GGUF Q8_0 bytes -> (q int8 [out, in], scale f16-bits uint16 [in/32, out]) on the host.

    The scales are k-block-major: scale[kb, n] belongs to quants q[n, 32*kb : 32*kb + 32]."""
    buf = np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray) else \
        np.ascontiguousarray(data, dtype=np.uint8)
    q = np.empty((out_features, in_features), np.int8)
    s = np.empty((in_features // 32, out_features), np.uint16)
    _lib.call("sp_q8_0_repack_host", buf.ctypes.data_as(ctypes.c_void_p), buf.size, out_features,
              in_features, q.ctypes.data_as(ctypes.c_void_p), s.ctypes.data_as(ctypes.c_void_p))
    return q, s


def dequantize_q8_0(q: torch.Tensor, scale: torch.Tensor, out_features: int, in_features: int,
                    dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Planar Q8_0 -> [out_features, in_features] float (quantized_matmul.rs:376)."""
    dev = require_cuda(q, scale)
    out = torch.empty((out_features, in_features), dtype=dtype, device=dev)
    _lib.call("sp_q8_0_dequant", ptr(q), ptr(scale), out_features, in_features, ptr(out),
              dtype_code(dtype), stream_ptr(dev))
    return out


def repack_q8_0(gguf: torch.Tensor, out_features: int, in_features: int):
    """Device repack of GGUF Q8_0 bytes already resident on the GPU (uint8 tensor)."""
    dev = require_cuda(gguf)
    q = torch.empty((out_features, in_features), dtype=torch.int8, device=dev)
    s = torch.empty((in_features // 32, out_features), dtype=torch.int16, device=dev)
    _lib.call("sp_q8_0_repack", ptr(gguf), gguf.numel(), out_features, in_features, ptr(q),
              ptr(s), stream_ptr(dev))
    return q, s


@dataclass(frozen=True)
class RopeEpilogue:
    """Rotary embedding applied in a projection GEMM's epilogue (rope.rs:145-170): columns
    [0, cols) are head_dim-wide heads whose (even, odd) pairs rotate by the angle of position
    ((row + pos_offset) // pos_div) % pos_mod.  `table` is f32 [positions, head_dim/2, 2] of
    (cos, sin), from `rope_pair_table`."""

    table: torch.Tensor
    cols: int
    head_dim: int
    pos_offset: int = 0
    pos_div: int = 1
    pos_mod: Optional[int] = None

    def args(self):
        mod = self.pos_mod if self.pos_mod is not None else self.table.shape[0]
        return (ptr(self.table), self.table.shape[0], self.cols, self.head_dim, self.pos_offset,
                self.pos_div, mod)


_NO_ROPE = (ptr(None), 0, 0, 0, 0, 1, 1)  # table, positions, cols, head_dim, off, div, mod


def rope_pair_table(cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """[positions, head_dim] cos / sin tables (each value repeated for its pair, rope.rs:60-94)
    -> f32 [positions, head_dim/2, 2] (cos, sin) pairs for RopeEpilogue."""
    return torch.stack((cos[:, ::2].float(), sin[:, ::2].float()), dim=-1).contiguous()


def _output_rows(out, M, N, dev, dtype=torch.bfloat16):
    """The GEMM output as rows of N values `ldy` apart (a column slice of a wider buffer is
    fine: the DiT attention writes its cross-stream k/v next to the self stream's).  dtype:
    bf16, or f16 for attention inputs that need its finer rounding."""
    if dtype not in (torch.bfloat16, torch.float16):
        raise ValueError("the strided-output epilogue writes bf16 or f16")
    if out is None:
        return torch.empty((M, N), dtype=dtype, device=dev), N
    if out.dtype != dtype:
        raise ValueError(f"out must be {dtype}")
    try:
        o2 = out.view(M, N)
    except RuntimeError as e:
        raise ValueError("out must be rows of the output width with a uniform row stride") from e
    if o2.stride(1) != 1:
        raise ValueError("out rows must be contiguous")
    return out, o2.stride(0)


GLU_GEGLU, GLU_SWIGLU = 0, 1  # sp_glu_kind


def interleave_rows(first: torch.Tensor, second: torch.Tensor, dim: int = 0) -> torch.Tensor:
    """Stack two equally shaped halves row-interleaved along `dim` ((first j, second j), ...),
    the weight layout of the GLU epilogue: [F, ...] + [F, ...] -> [2F, ...]."""
    return torch.stack((first, second), dim=dim + 1).flatten(dim, dim + 1)


def _epilogue_operands(gate, residual, M, N):
    """bf16 gate [N] and residual [M, N] (contiguous rows) for the gated-residual epilogue."""
    g = None
    if gate is not None:
        g = gate.reshape(-1)
        if g.numel() != N:
            raise ValueError(f"gate must hold {N} values")
        g = (g if g.dtype == torch.bfloat16 else g.to(torch.bfloat16)).contiguous()
    r = None
    if residual is not None:
        if residual.dtype != torch.bfloat16 or residual.numel() != M * N or not residual.is_contiguous():
            raise ValueError("residual must be a contiguous bf16 tensor of the output's shape")
        r = residual
    return g, r


class GpuQuantizedLinear:
    """quantized_matmul.rs:655-767: output = input @ weight.T (+ optional bias).

    Q8_0: q int8 [out, in], scale f16 bits [in/32, out].  K-quants: q = qpack uint8
    [out, in/2], scale = a and kmin = b, f32 [in/sub, out]."""

    def __init__(self, q: torch.Tensor, scale: torch.Tensor, out_features: int, in_features: int,
                 dtype: torch.dtype = torch.bfloat16, bias: Optional[torch.Tensor] = None,
                 quant_type: GpuQuantType = GpuQuantType.Q8_0,
                 kmin: Optional[torch.Tensor] = None):
        self.q, self.scale, self.kmin = q, scale, kmin
        self.quant_type = quant_type
        if quant_type != GpuQuantType.Q8_0 and kmin is None:
            raise ValueError("k-quant layers need both factor arrays (scale = a, kmin = b)")
        self.out_features, self.in_features = out_features, in_features
        self.dtype = dtype
        self.bias = bias

    @classmethod
    def from_bytes(cls, data, quant_type: GpuQuantType, out_features: int, in_features: int,
                   device="cuda", dtype: torch.dtype = torch.bfloat16, bias=None):
        """Upload raw GGUF bytes (little-endian Q8_0 blocks or K-quant super-blocks), repacked
        losslessly."""
        if quant_type in _KQ:
            qp, a, b = repack_kquant_host(data, quant_type, out_features, in_features)
            t = lambda v: torch.from_numpy(v).to(device)  # noqa: E731
            return cls(t(qp), t(a), out_features, in_features, dtype, bias, quant_type, t(b))
        if quant_type != GpuQuantType.Q8_0:
            raise ValueError(f"{quant_type} is not supported")
        q, s = repack_q8_0_host(data, out_features, in_features)
        return cls(torch.from_numpy(q).to(device), torch.from_numpy(s.view(np.int16)).to(device),
                   out_features, in_features, dtype, bias)

    def dequantize(self, dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        if self.quant_type in _KQ:
            return dequantize_kquant(self.quant_type, self.q, self.scale, self.kmin,
                                     self.out_features, self.in_features, dtype or torch.float32)
        return dequantize_q8_0(self.q, self.scale, self.out_features, self.in_features,
                               dtype or torch.float32)

    def forward(self, input: torch.Tensor, out: Optional[torch.Tensor] = None,
                gate: Optional[torch.Tensor] = None,
                residual: Optional[torch.Tensor] = None,
                rope: Optional[RopeEpilogue] = None, glu: Optional[int] = None,
                out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """[..., in_features] -> [..., out_features] via the fused dequant-GEMM (bf16).

        With gate ([out_features]) and/or residual ([..., out_features], bf16, may be `out`),
        returns residual + gate * (input . W^T + bias) from the GEMM epilogue; with `rope`,
        the rotary embedding of its columns (and `out` may be a column slice of a wider
        buffer); with `glu` (GLU_SWIGLU / GLU_GEGLU, rows interleaved by `interleave_rows`),
        the gated [..., out_features / 2] feed-forward activation."""
        dev = require_cuda(input, self.q, gate, residual, None if rope is None else rope.table)
        lead = input.shape[:-1]
        x = input.reshape(-1, self.in_features)
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        x = x.contiguous()
        M = x.shape[0]
        b = self.bias
        if b is not None and b.dtype != torch.bfloat16:
            b = b.to(torch.bfloat16)
        if glu is not None:
            if self.quant_type != GpuQuantType.Q8_0 or gate is not None or residual is not None \
                    or rope is not None:
                raise ValueError("the GLU epilogue is for Q8_0 layers without gate/residual/rope")
            half = self.out_features // 2
            y = out if out is not None else torch.empty((M, half), dtype=torch.bfloat16, device=dev)
            if y.dtype != torch.bfloat16 or not y.is_contiguous() or y.numel() != M * half:
                raise ValueError("out must be a contiguous bf16 tensor of [..., out_features / 2]")
            _lib.call("sp_q8_0_linear_glu", ptr(x), ptr(self.q), ptr(self.scale), ptr(b), ptr(y),
                      M, self.out_features, self.in_features, int(glu), _lib.SP_BF16,
                      stream_ptr(dev))
            return y.reshape(*lead, half)
        if self.quant_type in _KQ:
            if gate is not None or residual is not None or rope is not None:
                raise ValueError("k-quant layers have the plain (bias) epilogue only")
            y = out if out is not None else torch.empty((M, self.out_features),
                                                        dtype=torch.bfloat16, device=dev)
            if y.dtype != torch.bfloat16 or not y.is_contiguous() or y.numel() != M * self.out_features:
                raise ValueError("out must be a contiguous bf16 tensor of the output's shape")
            _lib.call("sp_kquant_linear", _KQ[self.quant_type][0], ptr(x), ptr(self.q),
                      ptr(self.scale), ptr(self.kmin), ptr(b), ptr(y), M, self.out_features,
                      self.in_features, _lib.SP_BF16, stream_ptr(dev))
            y = y.reshape(*lead, self.out_features)
            return y if input.dtype == torch.bfloat16 else y.to(input.dtype)
        f16_out = out_dtype == torch.float16 or (out is not None and out.dtype == torch.float16)
        if rope is not None or f16_out or (out is not None and not out.is_contiguous()):
            if gate is not None or residual is not None:
                raise ValueError("the rope / strided-output epilogue takes no gate or residual")
            ydt = torch.float16 if f16_out else torch.bfloat16
            y, ldy = _output_rows(out, M, self.out_features, dev, ydt)
            r = rope.args() if rope is not None else _NO_ROPE
            _lib.call("sp_q8_0_linear_rope", ptr(x), ptr(self.q), ptr(self.scale), ptr(b), ptr(y),
                      ldy, M, self.out_features, self.in_features, *r,
                      _lib.SP_F16 if f16_out else _lib.SP_BF16, stream_ptr(dev))
            return y if out is not None else y.reshape(*lead, self.out_features)
        y = out if out is not None else torch.empty((M, self.out_features), dtype=torch.bfloat16,
                                                    device=dev)
        if gate is None and residual is None:
            _lib.call("sp_q8_0_linear", ptr(x), ptr(self.q), ptr(self.scale), ptr(b), ptr(y), M,
                      self.out_features, self.in_features, _lib.SP_BF16, stream_ptr(dev))
        else:
            g, r = _epilogue_operands(gate, residual, M, self.out_features)
            _lib.call("sp_q8_0_linear_gated", ptr(x), ptr(self.q), ptr(self.scale), ptr(b),
                      ptr(g), ptr(r), ptr(y), M, self.out_features, self.in_features,
                      _lib.SP_BF16, stream_ptr(dev))
        y = y.reshape(*lead, self.out_features)
        return y if input.dtype == torch.bfloat16 else y.to(input.dtype)

    forward_burn = forward
    __call__ = forward


def set_tile_pairing(enabled: bool) -> bool:
    """Process-wide tile mode of the quantized linears (sp_quant_linear_set_pairing): True runs
    two-CTA clusters per 512 x 256 tile (tcgen05.mma.cta_group::2) when M > 256; False (the
    default) one CTA per 256 x 256 tile.  Results are bit-identical.  Returns the old mode."""
    rc = _lib.load().sp_quant_linear_set_pairing(1 if enabled else 0)
    if rc < 0:
        raise _lib.SketchpadError("sp_quant_linear_set_pairing", rc, _lib.load().sp_last_error().decode())
    return bool(rc)


def q8_0_quantize_reference(w: np.ndarray) -> bytes:
    """GGUF Q8_0 encoder for building test/bench weights (ggml's scheme: per 32 values,
    d = absmax/127 stored as f16, q = round(v/d)).  Used only to make synthetic inputs."""
    w = np.asarray(w, np.float32).reshape(-1, 32)
    amax = np.abs(w).max(axis=1)
    d = (amax / 127.0).astype(np.float32)
    d16 = d.astype(np.float16)
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1), 0).astype(np.float32)
    q = np.clip(np.rint(w * inv[:, None]), -128, 127).astype(np.int8)
    out = np.empty((w.shape[0], 34), np.uint8)
    out[:, :2] = d16.view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def make_kquant_synthetic(quant_type: GpuQuantType, out_features: int, in_features: int,
                          seed: int = 0) -> bytes:
    """Random K-quant super-blocks: every quant / scale / mask byte uniform, d and dmin f16
    ~ U(0.0005, 0.005) (normal f16 values), so decoded weights are O(0.1)."""
    fmt, nbytes, _ = _KQ[quant_type]
    rng = np.random.default_rng(seed)
    nb = out_features * in_features // 256
    blocks = rng.integers(0, 256, (nb, nbytes), dtype=np.uint8)
    f16 = lambda: rng.uniform(0.0005, 0.005, nb).astype(np.float16).view(np.uint8).reshape(-1, 2)  # noqa: E731
    if quant_type == GpuQuantType.Q4K:
        blocks[:, 0:2], blocks[:, 2:4] = f16(), f16()
    elif quant_type == GpuQuantType.Q2K:
        blocks[:, 80:82], blocks[:, 82:84] = f16(), f16()
    else:
        blocks[:, 108:110] = f16()
    return blocks.tobytes()


def make_q8_0_synthetic(out_features: int, in_features: int, seed: int = 0) -> bytes:
    """BASELINE config 4's weights: int8 ~ U[-127,127], f16 scale ~ U(0.001, 0.02)."""
    rng = np.random.default_rng(seed)
    nb = out_features * in_features // 32
    blocks = np.empty((nb, 34), np.uint8)
    blocks[:, :2] = rng.uniform(0.001, 0.02, nb).astype(np.float16).view(np.uint8).reshape(-1, 2)
    blocks[:, 2:] = rng.integers(-127, 128, (nb, 32), dtype=np.int8).view(np.uint8)
    return blocks.tobytes()


__all__ = ["GpuQuantType", "GpuQuantizedLinear", "dequantize_q8_0", "repack_q8_0", "set_tile_pairing",
           "repack_q8_0_host", "q8_0_quantize_reference", "make_q8_0_synthetic",
           "repack_kquant_host", "dequantize_kquant", "make_kquant_synthetic"]
