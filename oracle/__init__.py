"""CPU oracle for the sketchpad denoiser hot path.

TEST INFRASTRUCTURE ONLY.  This package wraps ``oracle/_build/liboracle.so``, a C++17/OpenMP
restatement of the reference's fp32 Burn-ndarray semantics (each C function cites the
reference file:line it follows).  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
legs of ``bench.py`` may import it, and only as the checker or the timed CPU baseline; the
product package ``sketchpad_b200`` never does.

Parity status: Q8_0 decode/matmul and FP8 scalar rounding are pinned to the reference's
golden vectors (``tests/golden``); GroupNorm and attention are "parity unpinned" (the
reference ships no golden vectors for them) and are pinned only to hand-computed answers
of the reference formulas.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None
_lock = threading.Lock()

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i64 = ctypes.c_int64


def build(force: bool = False) -> str:
    """Compile liboracle.so with oracle/Makefile (idempotent)."""
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(
        os.path.getmtime(os.path.join(_HERE, f)) for f in ("oracle.cpp", "oracle.h")
    ):
        subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_LIB_PATH)
            L.or_set_threads.argtypes = [ctypes.c_int]
            L.or_set_threads.restype = ctypes.c_int
            L.or_get_threads.restype = ctypes.c_int
            L.or_f16_to_f32.argtypes = [_u16p, _f32p, _i64]
            L.or_f32_to_f16.argtypes = [_f32p, _u16p, _i64]
            L.or_groupnorm_act.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64,
                                           _i64, ctypes.c_float, ctypes.c_int]
            L.or_groupnorm_act_dtype.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64,
                                                 _i64, _i64, ctypes.c_float, ctypes.c_int,
                                                 ctypes.c_int]
            L.or_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64,
                                       _i64, ctypes.c_int, ctypes.c_float, ctypes.c_int]
            L.or_q8_0_dequantize.argtypes = [_u8p, _i64, _f32p]
            L.or_q8_0_matmul.argtypes = [_u8p, _i64, _i64, _f32p, _i64, _f32p]
            L.or_kquant_dequantize.argtypes = [ctypes.c_int, _u8p, _i64, _f32p]
            L.or_fp8_quantize_scalar.argtypes = [ctypes.c_float, ctypes.c_int]
            L.or_fp8_quantize_scalar.restype = ctypes.c_float
            L.or_fp8_quantize.argtypes = [_f32p, _i64, _i64, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_float, _f32p, _f32p]
            L.or_fp8_dequantize.argtypes = [_f32p, _f32p, _i64, _i64, _i64, _f32p]
            L.or_linear_nt.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64]
            L.or_linear_kn.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64]
            L.or_layernorm.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, ctypes.c_float]
            L.or_activation.argtypes = [_f32p, _f32p, _i64, ctypes.c_int]
            L.or_conv2d.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64,
                                    _i64, _i64, _i64, _i64]
            _lib = L
    return _lib


def _f(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_f32p)


def _check(rc, name):
    if rc != 0:
        raise ValueError(f"oracle {name} rejected its arguments (status {rc})")


def set_threads(n: int) -> int:
    return lib().or_set_threads(int(n))


def get_threads() -> int:
    return lib().or_get_threads()


def f16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    out = np.empty(b.shape, np.float32)
    lib().or_f16_to_f32(b.ctypes.data_as(_u16p), out.ctypes.data_as(_f32p), b.size)
    return out


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    a, p = _f(x)
    out = np.empty(a.shape, np.uint16)
    lib().or_f32_to_f16(p, out.ctypes.data_as(_u16p), a.size)
    return out


_GN_DTYPES = {None: 0, "f32": 0, "f16": 1, "bf16": 2}


def groupnorm_act(x, gamma, beta, num_groups: int = 32, eps: float = 1e-5, silu: bool = True,
                  dtype=None):
    """GroupNorm(+SiLU) of groupnorm.rs:62-102.  dtype None/"f32": the f32 path; "f16" /
    "bf16": x, gamma and beta are that dtype's values (given as f32) and the reference's
    cast back before the affine, and its f16/bf16 affine, clamp and SiLU, are rounded as the
    reference rounds them."""
    x, px = _f(x)
    g, pg = _f(gamma)
    b, pb = _f(beta)
    B, C, H, W = x.shape
    y = np.empty_like(x)
    _check(lib().or_groupnorm_act_dtype(px, pg, pb, y.ctypes.data_as(_f32p), B, C, H, W,
                                        num_groups, eps, 1 if silu else 0, _GN_DTYPES[dtype]),
           "groupnorm_act")
    return y


def attention(q, k, v, mask=None, causal=False, scale=0.0, variant=0):
    """q [..., Sq, D], k [..., Skv, D], v [..., Skv, Dv] -> [..., Sq, Dv]."""
    q, pq = _f(q)
    k, pk = _f(k)
    v, pv = _f(v)
    lead = q.shape[:-2]
    Sq, D = q.shape[-2:]
    Skv, Dv = v.shape[-2:]
    BH = int(np.prod(lead)) if lead else 1
    out = np.empty(lead + (Sq, Dv), np.float32)
    pm = None
    if mask is not None:
        mask, pm = _f(mask)
    _check(lib().or_attention(pq, pk, pv, pm, out.ctypes.data_as(_f32p), BH, Sq, Skv, D, Dv,
                              1 if causal else 0, float(scale), int(variant)), "attention")
    return out


def q8_0_dequantize(data: np.ndarray, n_elements: int) -> np.ndarray:
    d = np.ascontiguousarray(data, dtype=np.uint8)
    nb = n_elements // 32
    if d.size < nb * 34:
        raise ValueError("Q8_0 data shorter than n_elements")
    out = np.empty(nb * 32, np.float32)
    _check(lib().or_q8_0_dequantize(d.ctypes.data_as(_u8p), nb, out.ctypes.data_as(_f32p)),
           "q8_0_dequantize")
    return out


KQUANT_BLOCK_BYTES = {10: 84, 11: 110, 12: 144}  # GGML type id -> bytes per 256 values


def kquant_dequantize(fmt: int, data: np.ndarray, n_elements: int) -> np.ndarray:
    """Q2_K (10) / Q3_K (11) / Q4_K (12) super-blocks -> f32 (gguf.rs:737-871)."""
    d = np.ascontiguousarray(data, dtype=np.uint8)
    nb = n_elements // 256
    if d.size < nb * KQUANT_BLOCK_BYTES[fmt]:
        raise ValueError("k-quant data shorter than n_elements")
    out = np.empty(nb * 256, np.float32)
    _check(lib().or_kquant_dequantize(int(fmt), d.ctypes.data_as(_u8p), nb,
                                      out.ctypes.data_as(_f32p)), "kquant_dequantize")
    return out


def q8_0_matmul(data: np.ndarray, out_features: int, in_features: int, x: np.ndarray):
    d = np.ascontiguousarray(data, dtype=np.uint8)
    x, px = _f(x)
    M = x.size // in_features
    y = np.empty((M, out_features), np.float32)
    _check(lib().or_q8_0_matmul(d.ctypes.data_as(_u8p), out_features, in_features, px, M,
                                y.ctypes.data_as(_f32p)), "q8_0_matmul")
    return y.reshape(x.shape[:-1] + (out_features,))


def fp8_quantize_scalar(v: float, fmt: int = 0) -> float:
    return float(lib().or_fp8_quantize_scalar(float(v), int(fmt)))


def fp8_quantize(w, fmt: int = 0, per_channel: bool = True, scale=None):
    w, pw = _f(w)
    rows, cols = w.shape
    data = np.empty_like(w)
    sc = np.empty(rows if per_channel else 1, np.float32)
    _check(lib().or_fp8_quantize(pw, rows, cols, fmt, 1 if per_channel else 0,
                                 0 if scale is None else 1, 0.0 if scale is None else float(scale),
                                 data.ctypes.data_as(_f32p), sc.ctypes.data_as(_f32p)),
           "fp8_quantize")
    return data, sc


def e4m3_bytes_to_f32(codes) -> np.ndarray:
    """Value of each e4m3 byte (crates/sketchpad-core/src/quantization.rs:311-368: 4 exponent
    bits with bias 7, 3 mantissa bits, smallest normal 2^-6, subnormal step 2^-9, max 448).
    Gives the f32 values the reference's simulated Fp8Tensor holds for the same grid points."""
    c = np.ascontiguousarray(codes, dtype=np.uint8).astype(np.int32)
    sign = np.where(c & 0x80, -1.0, 1.0).astype(np.float32)
    e = (c >> 3) & 0xF
    m = (c & 0x7).astype(np.float32)
    normal = np.ldexp(1.0 + m / 8.0, e - 7).astype(np.float32)
    sub = (m * np.float32(2.0 ** -9)).astype(np.float32)
    v = np.where(e == 0, sub, normal).astype(np.float32) * sign
    return np.where((e == 0xF) & (c & 0x7 == 0x7), np.float32(np.nan), v).astype(np.float32)


def fp8_dequantize(data, scale):
    data, pd = _f(data)
    scale, ps = _f(scale)
    rows, cols = data.shape
    out = np.empty_like(data)
    _check(lib().or_fp8_dequantize(pd, ps, scale.size, rows, cols, out.ctypes.data_as(_f32p)),
           "fp8_dequantize")
    return out


def linear_nt(x, w_nk, b=None):
    x, px = _f(x)
    w, pw = _f(w_nk)
    N, K = w.shape
    M = x.size // K
    pb = None
    if b is not None:
        b, pb = _f(b)
    y = np.empty((M, N), np.float32)
    _check(lib().or_linear_nt(px, pw, pb, y.ctypes.data_as(_f32p), M, K, N), "linear_nt")
    return y.reshape(x.shape[:-1] + (N,))


def linear_kn(x, w_kn, b=None):
    x, px = _f(x)
    w, pw = _f(w_kn)
    K, N = w.shape
    M = x.size // K
    pb = None
    if b is not None:
        b, pb = _f(b)
    y = np.empty((M, N), np.float32)
    _check(lib().or_linear_kn(px, pw, pb, y.ctypes.data_as(_f32p), M, K, N), "linear_kn")
    return y.reshape(x.shape[:-1] + (N,))


def layernorm(x, gamma, beta, eps: float = 1e-5):
    x, px = _f(x)
    g, pg = _f(gamma)
    b, pb = _f(beta)
    n = x.shape[-1]
    y = np.empty_like(x)
    _check(lib().or_layernorm(px, pg, pb, y.ctypes.data_as(_f32p), x.size // n, n, eps),
           "layernorm")
    return y


def activation(x, kind: str):
    x, px = _f(x)
    y = np.empty_like(x)
    _check(lib().or_activation(px, y.ctypes.data_as(_f32p), x.size,
                               {"silu": 0, "gelu": 1, "sigmoid": 2}[kind]), "activation")
    return y


def conv2d(x, w, b=None, stride: int = 1, pad: int = 0):
    x, px = _f(x)
    w, pw = _f(w)
    B, Cin, H, W = x.shape
    Cout, _, kh, kw = w.shape
    Ho = (H + 2 * pad - kh) // stride + 1
    Wo = (W + 2 * pad - kw) // stride + 1
    pb = None
    if b is not None:
        b, pb = _f(b)
    y = np.empty((B, Cout, Ho, Wo), np.float32)
    _check(lib().or_conv2d(px, pw, pb, y.ctypes.data_as(_f32p), B, Cin, H, W, Cout, kh, kw,
                           stride, pad), "conv2d")
    return y


# ---- denoising-loop latent updates (numpy f32, one rounding per operation, reference order)
def _guided(eps_u, eps_c, g):
    # crates/sketchpad-samplers/src/ddim.rs:158-164: uncond + (cond - uncond) * scale
    u = np.asarray(eps_u, np.float32)
    if eps_c is None:
        return u
    return u + (np.asarray(eps_c, np.float32) - u) * np.float32(g)


def ddim_step(x, eps_u, eps_c, guidance, sqrt_one_minus_at, sqrt_at, sqrt_at_prev, dir_xt,
              noise=None, sigma=0.0):
    """crates/sketchpad-samplers/src/ddim.rs:96-133 with the step's scalars given."""
    f = np.float32
    eps = _guided(eps_u, eps_c, guidance)
    px0 = (np.asarray(x, f) - eps * f(sqrt_one_minus_at)) / f(sqrt_at)
    prev = px0 * f(sqrt_at_prev) + f(dir_xt) * eps
    if noise is not None:
        prev = prev + np.asarray(noise, f) * f(sigma)
    return prev


def dpmpp_2m_step(x, eps_u, eps_c, guidance, sigma, ratio, one_minus_exp_neg_h, prev=None,
                  one_plus_coeff=1.0, coeff=0.0):
    """crates/sketchpad-samplers/src/dpm.rs:126-165: returns (next latent, denoised)."""
    f = np.float32
    eps = _guided(eps_u, eps_c, guidance)
    xv = np.asarray(x, f)
    den = xv - eps * f(sigma)
    d = den if prev is None else den * f(one_plus_coeff) - np.asarray(prev, f) * f(coeff)
    return xv * f(ratio) + d * f(one_minus_exp_neg_h), den

