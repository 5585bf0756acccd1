"""Weight files -> the GPU layers: GGUF Q8_0 / K-quant tensors into GpuQuantizedLinear and
safetensors F8_E4M3 tensors into Fp8Linear, through the library's native readers
(sp_model_* in include/sketchpad_b200.h: memory-mapped, host only).

Follows rhi-zone/sketchpad:
  crates/sketchpad-convert/src/gguf.rs:351-470   GgufFile::open / tensor_raw_data (GGUF v3,
                                                  32-byte data alignment, shapes reversed to
                                                  row-major [out_features, in_features])
  crates/sketchpad-convert/src/loader.rs:60-170   SafeTensorFile::open / load_f32 (F32, F16,
                                                  BF16 converted to f32 exactly)
  crates/sketchpad-cubecl/src/quantized_matmul.rs:670-702   GpuQuantizedLinear::from_bytes
  crates/sketchpad-core/src/quantization.rs:587-615         Fp8Linear
The reference's safetensors reader has no FP8 dtype; F8_E4M3 weights (with an f32 scale
tensor, per output channel or per tensor) are this library's addition for the FP8 linears.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple, Union

import numpy as np
import torch

from . import _lib

CONTAINER_GGUF, CONTAINER_SAFETENSORS = 1, 2
T_F32, T_F16, T_BF16, T_F8_E4M3, T_F8_E5M2, T_F64 = 0, 1, 2, 3, 4, 5
T_I8, T_U8, T_I16, T_I32, T_I64, T_BOOL = 6, 7, 8, 9, 10, 11
T_GGML_BASE = 100
GGML_Q8_0, GGML_Q2_K, GGML_Q3_K, GGML_Q4_K = 8, 10, 11, 12


@dataclass(frozen=True)
class TensorInfo:
    name: str
    type: int            # sp_tensor_type
    shape: Tuple[int, ...]  # row-major
    nbytes: int
    index: int

    @property
    def ggml_type(self) -> Optional[int]:
        """The ggml type id of a GGUF tensor (0 F32, 1 F16, 8 Q8_0, 12 Q4_K, ...)."""
        if self.type >= T_GGML_BASE:
            return self.type - T_GGML_BASE
        return {T_F32: 0, T_F16: 1}.get(self.type)


class ModelFile:
    """A GGUF or safetensors file opened by the native reader (the container is detected by
    the GGUF magic).  Tensor bytes are zero-copy views of the memory map, valid while open."""

    def __init__(self, path: str):
        self._L = _lib.load()
        self._h = ctypes.c_void_p()
        _lib.call("sp_model_open", str(path).encode(), ctypes.byref(self._h))
        c, nt, nm = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
        _lib.call("sp_model_info", self._h, ctypes.byref(c), ctypes.byref(nt), ctypes.byref(nm))
        self.container = c.value
        self.metadata_keys: List[str] = []
        buf = ctypes.create_string_buffer(4096)
        for i in range(nm.value):
            _lib.call("sp_model_meta_key", self._h, i, buf, len(buf))
            self.metadata_keys.append(buf.value.decode())
        self.tensors: Dict[str, TensorInfo] = {}
        t, nd, nb = ctypes.c_int(), ctypes.c_int(), ctypes.c_uint64()
        dims = (ctypes.c_int64 * 8)()
        for i in range(nt.value):
            _lib.call("sp_model_tensor_info", self._h, i, buf, len(buf), ctypes.byref(t),
                      ctypes.byref(nd), dims, ctypes.byref(nb))
            name = buf.value.decode()
            self.tensors[name] = TensorInfo(name, t.value, tuple(dims[:nd.value]), nb.value, i)

    # -- access ------------------------------------------------------------------------------
    def close(self) -> None:
        if self._h:
            _lib.call("sp_model_close", self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:  # pragma: no cover - interpreter shutdown
            pass

    def info(self, name: str) -> TensorInfo:
        try:
            return self.tensors[name]
        except KeyError:
            raise KeyError(f"tensor '{name}' not found") from None

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes as a read-only uint8 view of the map (gguf.rs tensor_raw_data)."""
        if not self._h:
            raise ValueError("the file is closed")
        info = self.info(name)
        p = ctypes.POINTER(ctypes.c_uint8)()
        _lib.call("sp_model_tensor_data", self._h, info.index, ctypes.byref(p))
        a = np.ctypeslib.as_array(p, shape=(info.nbytes,))
        a.flags.writeable = False
        return a

    def load_f32(self, name: str, device="cpu") -> torch.Tensor:
        """SafeTensorFile::load_f32 (loader.rs:112-170): F32 / F16 / BF16 -> f32, exactly."""
        info = self.info(name)
        raw = self.raw(name)
        if info.type == T_F32:
            a = raw.view("<f4")
        elif info.type == T_F16:
            a = raw.view("<f2").astype(np.float32)
        elif info.type == T_BF16:
            a = (raw.view("<u2").astype(np.uint32) << 16).view(np.float32)
        else:
            raise TypeError(f"tensor '{name}': type {info.type} is not F32, F16 or BF16")
        return torch.from_numpy(np.array(a, np.float32).reshape(info.shape)).to(device)

    # -- layers ------------------------------------------------------------------------------
    def quantized_linear(self, name: str, bias: Optional[torch.Tensor] = None, device="cuda"):
        """GpuQuantizedLinear::from_bytes over a GGUF Q8_0 / Q4_K / Q2_K / Q3_K weight
        [out_features, in_features] (rows of GGUF blocks, passed to the repack unchanged)."""
        from .quantized_matmul import GpuQuantizedLinear, GpuQuantType
        info = self.info(name)
        qt = {GGML_Q8_0: GpuQuantType.Q8_0, GGML_Q4_K: GpuQuantType.Q4K,
              GGML_Q2_K: GpuQuantType.Q2K, GGML_Q3_K: GpuQuantType.Q3K}.get(info.ggml_type)
        if self.container != CONTAINER_GGUF or qt is None or len(info.shape) != 2:
            raise TypeError(f"tensor '{name}' is not a 2-D GGUF Q8_0 / K-quant weight")
        out_f, in_f = info.shape
        b = None if bias is None else bias.to(device=device, dtype=torch.bfloat16).contiguous()
        return GpuQuantizedLinear.from_bytes(self.raw(name).tobytes(), qt, out_f, in_f,
                                             device=device, bias=b)

    def fp8_linear(self, name: str, scale: Union[str, float, None] = None,
                   bias: Union[str, torch.Tensor, None] = None, device="cuda"):
        """Fp8Linear from a safetensors F8_E4M3 weight [N, K]: `scale` names an f32 tensor of
        N (per output channel) or 1 values, or is a float; `bias` names a tensor (F32 / F16 /
        BF16, N values) or is one."""
        from .quantization import Fp8Format, Fp8Linear, Fp8Tensor
        info = self.info(name)
        if info.type != T_F8_E4M3 or len(info.shape) != 2:
            raise TypeError(f"tensor '{name}' is not a 2-D F8_E4M3 weight")
        N, K = info.shape
        if scale is None:
            s = torch.ones(1)
        elif isinstance(scale, str):
            s = self.load_f32(scale).reshape(-1)
            if s.numel() not in (1, N):
                raise ValueError(f"scale '{scale}' has {s.numel()} values; expected 1 or {N}")
        else:
            s = torch.tensor([float(scale)])
        data = torch.from_numpy(np.array(self.raw(name))).reshape(N, K).to(device)
        b = self.load_f32(bias) if isinstance(bias, str) else bias
        if b is not None:
            b = b.reshape(-1).to(device=device, dtype=torch.bfloat16)
        return Fp8Linear(Fp8Tensor(data, s.to(device, torch.float32).contiguous(), Fp8Format.E4M3,
                                   (N, K)), b)


__all__ = ["ModelFile", "TensorInfo", "CONTAINER_GGUF", "CONTAINER_SAFETENSORS"]
