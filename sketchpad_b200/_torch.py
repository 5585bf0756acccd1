"""torch plumbing for the ctypes calls: dtype codes, stream handles, pointer extraction."""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_DT = {torch.float32: _lib.SP_F32, torch.float16: _lib.SP_F16, torch.bfloat16: _lib.SP_BF16}


def dtype_code(t: torch.dtype) -> int:
    try:
        return _DT[t]
    except KeyError:
        raise TypeError(f"unsupported dtype {t}; expected float32, float16 or bfloat16") from None


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("sketchpad_b200 ops take CUDA tensors (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def stream_ptr(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def strides4(t: torch.Tensor):
    return _lib.i64_array(t.stride())
