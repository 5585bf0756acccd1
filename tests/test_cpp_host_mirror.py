"""The C++ host mirror (include/sketchpad_b200.hpp) over the C ABI: the reference's operators
for compiled callers, with the reference's names and error behaviour.

  * setup errors (CPU): attention shape / dtype / mask errors raise AttentionSetupError
    (attention.rs:97-104 returns Err there), GroupNorm and the quantized layers reject bad
    shapes before any device call;
  * parity (GPU): attention with a 77-key tail, GroupNorm+SiLU f32, LayerNorm f32, a Q8_0 and
    an FP8 linear run through the C++ operators on seeded inputs, checked against the CPU
    oracle.
"""
import os
import shutil
import subprocess

import numpy as np
import pytest

import oracle
from helpers import TOL_F32, TOL_HALF, rel_err

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _compile(name, tmp_path):
    gxx = shutil.which("g++")
    if gxx is None or not os.path.isdir(os.path.join(CUDA, "include")):
        pytest.skip("g++ or the CUDA headers are not available")
    from sketchpad_b200 import build as _build
    try:
        lib = _build.build()
    except RuntimeError as exc:  # no nvcc on this machine: nothing to link against
        if "nvcc not found" in str(exc):
            pytest.skip(str(exc))
        raise
    exe = str(tmp_path / name)
    libdir = os.path.dirname(lib)
    cmd = [gxx, "-std=c++17", "-O1", "-Wall", "-I" + os.path.join(ROOT, "include"),
           "-I" + os.path.join(CUDA, "include"), os.path.join(ROOT, "tests", "cpp", name + ".cpp"),
           "-L" + libdir, "-lsketchpad_b200", "-L" + os.path.join(CUDA, "lib64"), "-lcudart",
           "-Wl,-rpath," + libdir, "-Wl,-rpath," + os.path.join(CUDA, "lib64"), "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_cpp_mirror_setup_errors(tmp_path):
    exe = _compile("host_mirror_errors", tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr


def _bf16(bits):
    return (np.asarray(bits, np.uint32) << 16).view(np.float32)


@pytest.mark.gpu
def test_cpp_mirror_parity(tmp_path):
    exe = _compile("host_mirror_parity", tmp_path)
    out = str(tmp_path / "arrays.bin")
    r = subprocess.run([exe, out], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    buf = open(out, "rb").read()
    pos = 0

    def take(dtype, count):
        nonlocal pos
        a = np.frombuffer(buf, dtype, count, pos)
        pos += a.nbytes
        return a

    # attention [1,2,200,64] x [1,2,77,64]
    q = _bf16(take(np.uint16, 2 * 200 * 64)).reshape(2, 200, 64)
    k = _bf16(take(np.uint16, 2 * 77 * 64)).reshape(2, 77, 64)
    v = _bf16(take(np.uint16, 2 * 77 * 64)).reshape(2, 77, 64)
    o = take(np.float32, 2 * 200 * 64).reshape(2, 200, 64)
    for h in range(2):
        assert rel_err(o[h], oracle.attention(q[h], k[h], v[h])) < 1e-2
    # GroupNorm + SiLU, f32
    x = take(np.float32, 2 * 64 * 16 * 16).reshape(2, 64, 16, 16)
    g = take(np.float32, 64)
    b = take(np.float32, 64)
    y = take(np.float32, 2 * 64 * 16 * 16).reshape(2, 64, 16, 16)
    assert rel_err(y, oracle.groupnorm_act(x, g, b, 32, 1e-5, True)) < TOL_F32
    # Q8_0 linear, 128 x 256 weights, x [64, 256]
    gguf = take(np.uint8, 128 * (256 // 32) * 34)
    xq = _bf16(take(np.uint16, 64 * 256)).reshape(64, 256)
    yq = _bf16(take(np.uint16, 64 * 128)).reshape(64, 128)
    assert rel_err(yq, oracle.q8_0_matmul(gguf, 128, 256, xq)) < TOL_HALF
    # LayerNorm f32 [64, 320]
    lx = take(np.float32, 64 * 320).reshape(64, 320)
    lg = take(np.float32, 320)
    lb = take(np.float32, 320)
    ly = take(np.float32, 64 * 320).reshape(64, 320)
    assert rel_err(ly, oracle.layernorm(lx, lg, lb, 1e-5)) < TOL_F32
    # FP8 linear, per-channel e4m3 weights
    w = take(np.float32, 128 * 256).reshape(128, 256)
    xf = _bf16(take(np.uint16, 64 * 256)).reshape(64, 256)
    yf = _bf16(take(np.uint16, 64 * 128)).reshape(64, 128)
    data, sc = oracle.fp8_quantize(w)
    assert rel_err(yf, oracle.linear_nt(xf, oracle.fp8_dequantize(data, sc))) < TOL_HALF
    # GroupNorm + SiLU, channels-last B = 1 with an unusual batch stride (gathered to NCHW
    # through the strides the mirror labelled y with)
    x1 = take(np.float32, 64 * 16 * 16).reshape(1, 64, 16, 16)
    g1 = take(np.float32, 64)
    b1 = take(np.float32, 64)
    y1 = take(np.float32, 64 * 16 * 16).reshape(1, 64, 16, 16)
    assert pos == len(buf)
    assert rel_err(y1, oracle.groupnorm_act(x1, g1, b1, 32, 1e-5, True)) < TOL_F32
