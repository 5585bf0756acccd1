"""The C-ABI library loads and exports every entry point include/sketchpad_b200.h declares,
and its host-only paths (argument checks, host repack) work without a GPU."""
import ctypes
import os
import re

import numpy as np

import oracle
from sketchpad_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    src = open(os.path.join(ROOT, "include", "sketchpad_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(sp_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    names = declared_functions()
    assert len(names) >= 14
    for n in names:
        assert hasattr(L, n), f"{n} declared in the header but not exported"
    assert set(names) == set(_lib.SIGNATURES), "ctypes binding and header disagree"


def test_abi_version():
    assert _lib.load().sp_abi_version() == 1


def test_groupnorm_rejects_indivisible_channels_without_touching_the_gpu():
    L = _lib.load()
    st = _lib.i64_array((30 * 4, 4, 2, 1))
    rc = L.sp_groupnorm_act(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16),
                            ctypes.c_void_p(16), 1, 30, 2, 2, st, 32, 1e-5, 1, 0, None, 0, None)
    assert rc == -2
    assert b"divisible" in L.sp_last_error()


def test_null_and_shape_errors_are_status_codes():
    L = _lib.load()
    s4 = _lib.i64_array((1, 1, 1, 1))
    assert L.sp_flash_attn_fwd(None, None, None, None, 0, None, 1, 1, 1, 1, 64, 64, s4, s4, s4, s4,
                               2, 2, 0, 0.0, None) == -1
    p = ctypes.c_void_p(256)
    assert L.sp_flash_attn_fwd(p, p, p, None, 0, p, 1, 1, 1, 1, 36, 36, s4, s4, s4, s4, 2, 2, 0,
                               0.0, None) == -2  # head dim not a multiple of 8
    assert L.sp_q8_0_linear(p, p, p, None, p, 4, 16, 48, 2, None) == -2  # K % 64
    assert L.sp_fp8_linear(p, p, p, 3, None, p, 4, 16, 64, 2, None) == -2  # scale count
    assert L.sp_layernorm(p, p, p, p, 4, 1, 1e-5, 1, 0, None) == -1


def test_q8_0_host_repack_matches_oracle_decode():
    rng = np.random.default_rng(0)
    out_f, in_f = 8, 96
    nb = out_f * in_f // 32
    blocks = np.empty((nb, 34), np.uint8)
    # include subnormal and negative f16 scales
    scales = rng.uniform(-0.02, 0.02, nb).astype(np.float16)
    scales[:3] = np.array([6e-8, -3e-6, 0.0], np.float16)
    blocks[:, :2] = scales.view(np.uint8).reshape(-1, 2)
    blocks[:, 2:] = rng.integers(-128, 128, (nb, 32), dtype=np.int8).view(np.uint8)
    raw = blocks.tobytes()
    q = np.empty((out_f, in_f), np.int8)
    s = np.empty((in_f // 32, out_f), np.uint16)
    buf = np.frombuffer(raw, np.uint8)
    rc = _lib.load().sp_q8_0_repack_host(buf.ctypes.data_as(ctypes.c_void_p), buf.size, out_f, in_f,
                                         q.ctypes.data_as(ctypes.c_void_p),
                                         s.ctypes.data_as(ctypes.c_void_p))
    assert rc == 0
    dec = oracle.f16_bits_to_f32(s.T).repeat(32, axis=1) * q.astype(np.float32)
    ref = oracle.q8_0_dequantize(buf, out_f * in_f).reshape(out_f, in_f)
    assert np.array_equal(dec.view(np.uint32), ref.view(np.uint32))


def test_ulysses_a2a_and_comm_argument_errors_without_a_gpu():
    # argument checks come before NCCL or the device is touched (include/sketchpad_b200.h)
    L = _lib.load()
    p = ctypes.c_void_p(256)
    assert L.sp_ulysses_a2a(p, ctypes.c_void_p(512), 16, 2, None, None, 1.0) == -1  # no comm
    assert L.sp_ulysses_a2a(p, ctypes.c_void_p(512), 0, 2, p, None, 1.0) == -1      # count
    assert L.sp_ulysses_a2a(p, ctypes.c_void_p(512), 16, 9, p, None, 1.0) == -3     # dtype
    assert L.sp_ulysses_a2a(p, p, 16, 2, p, None, 1.0) == -1                         # aliasing
    assert b"alias" in L.sp_last_error()
    assert L.sp_ulysses_a2a(p, ctypes.c_void_p(512), 16, 2, p, None, 0.0) == -1     # deadline
    comm = ctypes.c_void_p()
    uid = ctypes.create_string_buffer(128)
    assert L.sp_nccl_comm_init(ctypes.byref(comm), 2, 2, uid, 1.0) == -1           # rank >= n
    assert L.sp_nccl_comm_init(ctypes.byref(comm), 2, 0, None, 1.0) == -1          # no id
    assert L.sp_nccl_comm_init(ctypes.byref(comm), 2, 0, uid, -1.0) == -1          # deadline
    assert L.sp_nccl_wait(None, None, 1.0) == -1
    assert L.sp_nccl_comm_abort(None) == -1
    assert L.sp_nccl_comm_destroy(None, 1.0) == -1


def test_nccl_unique_id_on_the_host():
    # the id is made on the host (NCCL bootstrap, no device): 128 bytes, fresh each call
    L = _lib.load()
    n = L.sp_nccl_unique_id_bytes()
    assert n == 128
    assert L.sp_nccl_unique_id(ctypes.create_string_buffer(8), 8) == -1
    a, b = ctypes.create_string_buffer(n), ctypes.create_string_buffer(n)
    rc = L.sp_nccl_unique_id(a, n)
    if rc == -8:  # no NCCL on this machine: the status says so
        assert b"NCCL" in L.sp_last_error()
        return
    assert rc == 0 and L.sp_nccl_unique_id(b, n) == 0
    assert a.raw != bytes(n) and a.raw != b.raw


def test_quant_linear_pairing_mode_switch_on_the_host():
    L = _lib.load()
    assert L.sp_quant_linear_set_pairing(2) == -1  # SP_ERR_INVALID_ARG
    old = L.sp_quant_linear_set_pairing(1)
    assert old in (0, 1)
    assert L.sp_quant_linear_set_pairing(old) == 1


def test_groupnorm_streaming_workspace_size_on_the_host():
    # contiguous NCHW groups of 256 KB and more take the streaming slice-unit path: the
    # workspace is one u32 counter per (batch, group), padded to 16 bytes, then a 16-byte
    # partial per slice unit (48 KB units for f32, 64 KB for 16-bit types)
    L = _lib.load()
    B, C, H, W, G = 8, 512, 128, 128, 32
    st = _lib.i64_array((C * H * W, H * W, W, 1))
    for dtype, es, unit in ((0, 4, 48 * 1024), (1, 2, 64 * 1024), (2, 2, 64 * 1024)):
        group_bytes = C // G * H * W * es
        S = -(-group_bytes // unit)
        BG = B * G
        want = ((BG * 4 + 15) // 16) * 16 + BG * S * 16
        assert L.sp_groupnorm_act_workspace_size(B, C, H, W, st, G, dtype) == want
