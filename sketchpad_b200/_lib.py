"""ctypes binding of libsketchpad_b200.so (the C ABI in include/sketchpad_b200.h).

There is no fallback: if the library is missing or the device is not sm_100, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsketchpad_b200.so")

SP_OK = 0
SP_F32, SP_F16, SP_BF16 = 0, 1, 2
SP_ACT_NONE, SP_ACT_SILU = 0, 1

_STATUS = {
    -1: "invalid argument", -2: "unsupported shape", -3: "unsupported dtype",
    -4: "alignment", -5: "launch failure", -6: "workspace", -7: "device is not sm_100",
    -8: "communication failure or deadline",
}

_lib = None
_lock = threading.Lock()

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i64p = ctypes.POINTER(ctypes.c_int64)
_int = ctypes.c_int
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); the single source of the binding, also used by the ABI test
SIGNATURES = {
    "sp_abi_version": (_int, []),
    "sp_last_error": (ctypes.c_char_p, []),
    "sp_watchdog_read_and_clear": (_int, [_vp, ctypes.POINTER(_int)]),
    "sp_flash_attn_fwd": (_int, [_vp, _vp, _vp, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64,
                                 _i64, _i64p, _i64p, _i64p, _i64p, _int, _int, _int, _f, _vp]),
    "sp_flash_attn_fwd_wait_test": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int,
                                           _i64, _vp]),
    "sp_bf16_linear": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "sp_bf16_linear_gated": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "sp_bf16_linear_glu": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _int, _vp]),
    "sp_groupnorm_act_workspace_size": (_sz, [_i64, _i64, _i64, _i64, _i64p, _i64, _int]),
    "sp_groupnorm_act_output_strides": (_int, [_i64, _i64, _i64, _i64, _i64p, _i64p]),
    "sp_model_open": (_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "sp_model_close": (_int, [_vp]),
    "sp_model_info": (_int, [_vp, ctypes.POINTER(_int), ctypes.POINTER(_i64), ctypes.POINTER(_i64)]),
    "sp_model_meta_key": (_int, [_vp, _i64, ctypes.c_char_p, _sz]),
    "sp_model_tensor_info": (_int, [_vp, _i64, ctypes.c_char_p, _sz, ctypes.POINTER(_int),
                                    ctypes.POINTER(_int), _i64p, ctypes.POINTER(ctypes.c_uint64)]),
    "sp_model_find": (_int, [_vp, ctypes.c_char_p, ctypes.POINTER(_i64)]),
    "sp_model_tensor_data": (_int, [_vp, _i64, ctypes.POINTER(ctypes.POINTER(ctypes.c_uint8))]),
    "sp_nccl_unique_id_bytes": (_sz, []),
    "sp_nccl_unique_id": (_int, [_vp, _sz]),
    "sp_nccl_comm_init": (_int, [ctypes.POINTER(_vp), _int, _int, _vp, ctypes.c_double]),
    "sp_nccl_comm_poll": (_int, [_vp, ctypes.POINTER(_int)]),
    "sp_nccl_wait": (_int, [_vp, _vp, ctypes.c_double]),
    "sp_nccl_comm_abort": (_int, [_vp]),
    "sp_nccl_comm_destroy": (_int, [_vp, ctypes.c_double]),
    "sp_ulysses_a2a": (_int, [_vp, _vp, _i64, _int, _vp, _vp, ctypes.c_double]),
    "sp_nccl_all_gather": (_int, [_vp, _vp, _i64, _int, _vp, _vp, ctypes.c_double]),
    "sp_groupnorm_act": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64p, _i64, _f,
                                _int, _int, _vp, _sz, _vp]),
    "sp_groupnorm_add_act": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64p,
                                    _i64, _f, _int, _int, _vp, _sz, _vp]),
    "sp_groupnorm_act_noalloc_max_scratch_bytes": (_sz, []),
    "sp_groupnorm_act_noalloc": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64p, _i64,
                                        _f, _int, _int, _vp]),
    "sp_glu_gate": (_int, [_vp, _vp, _i64, _i64, _i64, _i64, _int, _int, _vp]),
    "sp_add_bias_residual": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _int, _vp]),
    "sp_q8_0_repack_host": (_int, [_vp, _sz, _i64, _i64, _vp, _vp]),
    "sp_q8_0_repack": (_int, [_vp, _sz, _i64, _i64, _vp, _vp, _vp]),
    "sp_q8_0_dequant": (_int, [_vp, _vp, _i64, _i64, _vp, _int, _vp]),
    "sp_q8_0_linear": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "sp_q8_0_linear_gated": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "sp_fp8_quantize": (_int, [_vp, _i64, _i64, _int, _vp, _vp, _vp]),
    "sp_fp8_dequant": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _int, _vp]),
    "sp_fp8_linear": (_int, [_vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "sp_fp8_linear_gated": (_int, [_vp, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int,
                                   _vp]),
    "sp_cfg_ddim_step": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _f, _f, _f, _f, _f, _f, _int, _vp]),
    "sp_cfg_dpmpp_2m_step": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _f, _f, _f, _f, _f, _f, _int,
                                    _int, _vp]),
    "sp_kquant_repack_host": (_int, [_int, _vp, _sz, _i64, _i64, _vp, _vp, _vp]),
    "sp_kquant_dequant": (_int, [_int, _vp, _vp, _vp, _i64, _i64, _vp, _int, _vp]),
    "sp_kquant_linear": (_int, [_int, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "sp_q8_0_linear_glu": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _int, _vp]),
    "sp_quant_linear_set_pairing": (_int, [_int]),
    "sp_fp8_linear_glu": (_int, [_vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _int, _int,
                                 _vp]),
    "sp_q8_0_linear_rope": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64,
                                   _i64, _i64, _i64, _i64, _i64, _int, _vp]),
    "sp_fp8_linear_rope": (_int, [_vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _vp,
                                  _i64, _i64, _i64, _i64, _i64, _i64, _int, _vp]),
    "sp_layernorm": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _f, _int, _int, _vp]),
    "sp_layernorm_add": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _f, _int, _int, _vp]),
    "sp_layernorm_modulate": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f, _int, _int,
                                     _vp]),
}


class SketchpadError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn}: {_STATUS.get(status, status)}: {msg}")
        self.status = status


def load():
    """Load (building first if this checkout has no library yet) and bind the library."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                from . import build as _build
                _build.build()
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def call(name: str, *args) -> int:
    rc = getattr(load(), name)(*args)
    if rc != SP_OK:
        raise SketchpadError(name, rc, load().sp_last_error().decode())
    return rc


def i64_array(vals):
    arr = (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])
    return arr
