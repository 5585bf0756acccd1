"""Q8_0 and FP8 weight paths vs the CPU oracle.

Dequantized weights: bit-exact (f32).  Linears (bf16 activations, bf16 output): rel_err =
max|gpu - oracle| / max|oracle| < 2e-2, the oracle running in fp32 on the same bf16 x.
"""
import numpy as np
import pytest
import torch

import oracle
from sketchpad_b200 import (Fp8Config, Fp8Linear, GpuQuantizedLinear, GpuQuantType,
                            dequantize_q8_0, quantize_fp8, repack_q8_0)
from sketchpad_b200.quantized_matmul import make_q8_0_synthetic, q8_0_quantize_reference
from sketchpad_b200.quantization import Fp8Tensor, Fp8Format
from helpers import TOL_HALF, rel_err, to_np

pytestmark = pytest.mark.gpu


def test_q8_0_golden_vectors_on_gpu():
    import json, os
    here = os.path.join(os.path.dirname(__file__), "golden")
    for name in ("q8_0_decode_scale_half", "q8_0_decode_known_values"):
        case = json.load(open(os.path.join(here, name + ".json")))
        raw = bytes.fromhex(case["bytes_hex"])
        lin = GpuQuantizedLinear.from_bytes(raw, GpuQuantType.Q8_0, 1, 32)
        got = to_np(lin.dequantize()).ravel()
        assert np.array_equal(got, np.array(case["expected"], np.float32))


def test_q8_0_dequant_bit_exact_with_subnormal_scales():
    out_f, in_f = 64, 256
    raw = bytearray(make_q8_0_synthetic(out_f, in_f, seed=1))
    blocks = np.frombuffer(raw, np.uint8).reshape(-1, 34).copy()
    blocks[:4, :2] = np.array([6e-8, -3e-6, 0.0, 1e-5], np.float16).view(np.uint8).reshape(-1, 2)
    raw = blocks.tobytes()
    ref = oracle.q8_0_dequantize(np.frombuffer(raw, np.uint8), out_f * in_f).reshape(out_f, in_f)
    lin = GpuQuantizedLinear.from_bytes(raw, GpuQuantType.Q8_0, out_f, in_f)
    got = to_np(lin.dequantize(torch.float32))
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    # device repack of GGUF bytes gives the same planar layout
    q, s = repack_q8_0(torch.frombuffer(bytearray(raw), dtype=torch.uint8).cuda(), out_f, in_f)
    assert torch.equal(q, lin.q) and torch.equal(s, lin.scale)
    got2 = to_np(dequantize_q8_0(q, s, out_f, in_f))
    assert np.array_equal(got2.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (200, 48, 128), (4608, 3072, 3072),
                                   (512, 9216, 3072), (77, 1280, 12288)])
def test_q8_0_linear_vs_oracle(M, N, K):
    raw = make_q8_0_synthetic(N, K, seed=M + N)
    lin = GpuQuantizedLinear.from_bytes(raw, GpuQuantType.Q8_0, N, K)
    g = torch.Generator(device="cpu").manual_seed(1)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    y = lin.forward(x.cuda())
    torch.cuda.synchronize()
    rows = slice(0, min(M, 256))  # the sequential-dot oracle is slow; check leading rows
    ref = oracle.q8_0_matmul(np.frombuffer(raw, np.uint8), N, K, to_np(x[rows]))
    assert rel_err(to_np(y[rows]), ref) < TOL_HALF
    if M > 256:
        ref_tail = oracle.q8_0_matmul(np.frombuffer(raw, np.uint8), N, K, to_np(x[-64:]))
        assert rel_err(to_np(y[-64:]), ref_tail) < TOL_HALF


def test_q8_0_linear_golden_2x32_padded():
    # quantized.rs:516-552: out = [~3, ~7]; N is padded to 16 rows of zero weights
    import json, os
    case = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "q8_0_matmul_2x32.json")))
    raw = bytes.fromhex(case["bytes_hex"])
    zero_blocks = bytes(34 * 14 * 2)  # 14 more rows of 64 values (2 blocks each)
    rows = []
    blocks = np.frombuffer(raw, np.uint8).reshape(2, 34)
    for r in range(2):  # widen each row to 64 values (K must be a multiple of 64)
        rows.append(blocks[r].tobytes() + bytes(34))
    full = b"".join(rows) + zero_blocks
    lin = GpuQuantizedLinear.from_bytes(full, GpuQuantType.Q8_0, 16, 64)
    x = torch.zeros(1, 64, dtype=torch.bfloat16)
    x[0, :32] = torch.tensor(case["input"])
    y = to_np(lin.forward(x.cuda()))[0]
    assert abs(y[0] - 3.0) < case["tol"] and abs(y[1] - 7.0) < case["tol"]
    assert np.all(y[2:] == 0)


def test_q8_0_linear_with_bias_3d():
    N, K = 256, 128
    raw = q8_0_quantize_reference(np.random.default_rng(2).standard_normal((N, K)).astype(np.float32))
    bias = torch.randn(N, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    lin = GpuQuantizedLinear.from_bytes(raw, GpuQuantType.Q8_0, N, K, bias=bias.cuda())
    x = torch.randn(2, 3, K, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16)
    y = lin.forward(x.cuda())
    assert y.shape == (2, 3, N)
    ref = oracle.q8_0_matmul(np.frombuffer(raw, np.uint8), N, K, to_np(x).reshape(6, K)) + to_np(bias)
    assert rel_err(to_np(y).reshape(6, N), ref) < TOL_HALF


def test_fp8_quantize_matches_reference_rounding():
    g = torch.Generator(device="cpu").manual_seed(5)
    w = torch.randn(64, 512, generator=g) * torch.rand(64, 1, generator=g) * 10
    fp8 = quantize_fp8(w.cuda(), Fp8Config.e4m3().with_per_channel(True))
    data_ref, scale_ref = oracle.fp8_quantize(w.numpy(), 0, True)
    assert np.array_equal(to_np(fp8.scale), scale_ref)
    deq = to_np(fp8.dequantize())
    deq_ref = oracle.fp8_dequantize(data_ref, scale_ref)
    # bit-exact wherever the reference's simulated value is on the e4m3 grid (|scaled| >= 2^-6)
    scaled = np.abs(w.numpy() / scale_ref[:, None])
    on_grid = scaled >= 2.0 ** -6
    assert on_grid.mean() > 0.99
    assert np.array_equal(deq[on_grid].view(np.uint32), deq_ref[on_grid].view(np.uint32))
    # below 2^-6 the e4m3 subnormal grid differs from the reference by < 2^-10 * scale
    off = ~on_grid
    assert np.all(np.abs(deq[off] - deq_ref[off]) <= (2.0 ** -10) * np.broadcast_to(scale_ref[:, None], deq.shape)[off] * 1.0001)


def test_fp8_per_tensor_and_explicit_scale():
    w = torch.tensor([[1.0, 2.0, 3.0, 4.0], [0.5, 1.5, 2.5, 3.5]])
    t = quantize_fp8(w.cuda(), Fp8Config.e4m3())
    d_ref, s_ref = oracle.fp8_quantize(w.numpy(), 0, False)
    assert np.array_equal(to_np(t.scale), s_ref)
    assert np.array_equal(to_np(t.dequantize()), oracle.fp8_dequantize(d_ref, s_ref))
    assert np.abs(to_np(t.dequantize()) - w.numpy()).max() < 0.5  # quantization.rs:815-831
    t2 = quantize_fp8(w.cuda(), Fp8Config.e4m3().with_scale(0.01))
    d2, s2 = oracle.fp8_quantize(w.numpy(), 0, False, scale=0.01)
    assert np.array_equal(to_np(t2.dequantize()), oracle.fp8_dequantize(d2, s2))


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 160, 320), (2048, 5120, 5120),
                                   (512, 13824, 5120), (256, 5120, 13824)])
def test_fp8_linear_vs_oracle(M, N, K):
    g = torch.Generator(device="cpu").manual_seed(M + K)
    w = torch.randn(N, K, generator=g) * 0.02
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    lin = Fp8Linear.from_weight(w.cuda(), bias.cuda(), Fp8Config.e4m3().with_per_channel(True))
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    y = lin.forward(x.cuda())
    torch.cuda.synchronize()
    wdq = to_np(lin.weight.dequantize())  # bit-exact decode (tested above)
    rows = slice(0, min(M, 256))
    ref = oracle.linear_nt(to_np(x[rows]), wdq, to_np(bias))
    assert rel_err(to_np(y[rows]), ref) < TOL_HALF


def test_fp8_synthetic_bytes_roundtrip():
    t = Fp8Tensor(torch.arange(256, dtype=torch.uint8).reshape(16, 16).cuda(),
                  torch.ones(16).cuda(), Fp8Format.E4M3, (16, 16))
    got = to_np(t.dequantize()).ravel()
    # e4m3 decode from the OCP bit layout, computed independently here
    exp = []
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e, m = (b >> 3) & 0xF, b & 7
        if e == 0xF and m == 7:
            exp.append(np.nan)
        elif e == 0:
            exp.append(s * m / 8 * 2.0 ** -6)
        else:
            exp.append(s * (1 + m / 8) * 2.0 ** (e - 7))
    exp = np.array(exp, np.float32)
    ok = ~np.isnan(exp)
    assert np.array_equal(got[ok], exp[ok]) and np.all(np.isnan(got[~ok]))


def _epilogue_ref(mm, gate, residual):
    # residual + gate * (x . W^T + b): Flux's `img + gate * proj(..)` (flux.rs:486-560) and
    # Wan's `x + to_out(..)` (wan.rs:430-470) in f32
    out = mm if gate is None else mm * gate[None, :]
    return out if residual is None else out + residual


@pytest.mark.parametrize("M,N,K", [(200, 256, 128), (4608, 3072, 3072), (77, 1536, 640),
                                   (512, 3072, 12288)])  # the last two run split-K
@pytest.mark.parametrize("mode", ["gate+residual", "residual", "gate", "in_place"])
def test_q8_0_linear_gated_residual_epilogue(M, N, K, mode):
    raw = make_q8_0_synthetic(N, K, seed=N + K)
    g = torch.Generator(device="cpu").manual_seed(M)
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    lin = GpuQuantizedLinear.from_bytes(raw, GpuQuantType.Q8_0, N, K, bias=bias.cuda())
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    gate = (torch.randn(N, generator=g)).to(torch.bfloat16) if mode != "residual" else None
    res = (torch.randn(M, N, generator=g) * 4).to(torch.bfloat16) if mode != "gate" else None
    rd = res.cuda() if res is not None else None
    y = lin.forward(x.cuda(), gate=None if gate is None else gate.cuda(), residual=rd,
                    out=rd if mode == "in_place" else None)
    torch.cuda.synchronize()
    if mode == "in_place":
        assert y.data_ptr() == rd.data_ptr()
    rows = slice(0, min(M, 256))
    mm = oracle.q8_0_matmul(np.frombuffer(raw, np.uint8), N, K, to_np(x[rows])) + to_np(bias)
    ref = _epilogue_ref(mm, None if gate is None else to_np(gate),
                        None if res is None else to_np(res[rows]))
    assert rel_err(to_np(y[rows]), ref) < TOL_HALF


@pytest.mark.parametrize("M,N,K", [(300, 160, 320), (2048, 5120, 5120)])
@pytest.mark.parametrize("in_place", [False, True])
def test_fp8_linear_residual_epilogue(M, N, K, in_place):
    g = torch.Generator(device="cpu").manual_seed(M + N)
    w = torch.randn(N, K, generator=g) * 0.02
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    lin = Fp8Linear.from_weight(w.cuda(), bias.cuda(), Fp8Config.e4m3().with_per_channel(True))
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    gate = torch.randn(N, generator=g).to(torch.bfloat16)
    res = (torch.randn(M, N, generator=g) * 4).to(torch.bfloat16)
    rd = res.cuda()
    y = lin.forward(x.cuda(), gate=gate.cuda(), residual=rd, out=rd if in_place else None)
    torch.cuda.synchronize()
    wdq = to_np(lin.weight.dequantize())
    rows = slice(0, min(M, 256))
    ref = _epilogue_ref(oracle.linear_nt(to_np(x[rows]), wdq, to_np(bias)), to_np(gate),
                        to_np(res[rows]))
    assert rel_err(to_np(y[rows]), ref) < TOL_HALF


def test_gated_epilogue_rejects_bad_operands():
    lin = GpuQuantizedLinear.from_bytes(make_q8_0_synthetic(64, 64, seed=1), GpuQuantType.Q8_0,
                                        64, 64)
    x = torch.randn(8, 64, device="cuda").to(torch.bfloat16)
    with pytest.raises(ValueError, match="gate"):
        lin.forward(x, gate=torch.ones(32, device="cuda"))
    with pytest.raises(ValueError, match="residual"):
        lin.forward(x, residual=torch.zeros(8, 64, device="cuda"))  # f32
    with pytest.raises(ValueError, match="residual"):
        lin.forward(x, residual=torch.zeros(64, 8, device="cuda", dtype=torch.bfloat16).t())


def _rope_ref(y, cos, sin, cols, D, off, div, mod):
    # rope.rs:145-170 per row of y [M, N] at position ((row + off) // div) % mod
    M = y.shape[0]
    pos = ((np.arange(M) + off) // div) % mod
    out = y.copy()
    h = y[:, :cols].reshape(M, cols // D, D)
    c, s = cos[pos][:, None, :], sin[pos][:, None, :]
    rot = np.stack((-h[..., 1::2], h[..., 0::2]), axis=-1).reshape(h.shape)
    out[:, :cols] = (h * c + rot * s).reshape(M, cols)
    return out


@pytest.mark.parametrize("M,N,K,D,off,div,mod", [
    (4608, 9216, 3072, 128, 0, 1, 4608),   # Flux qkv: q and k of 24 heads rotated
    (300, 384, 256, 64, 36, 24, 3),        # Wan temporal-style positions with a rank offset
    (77, 256, 128, 128, 5, 1, 40),
    (77, 512, 2048, 128, 3, 1, 100)])     # small grid: split-K, the epilogue in the reduce pass
def test_q8_0_linear_rope_epilogue_strided(M, N, K, D, off, div, mod):
    from sketchpad_b200.flux import rope_tables
    from sketchpad_b200.quantized_matmul import RopeEpilogue, rope_pair_table
    raw = make_q8_0_synthetic(N, K, seed=N + 7)
    g = torch.Generator(device="cpu").manual_seed(M + 3)
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    lin = GpuQuantizedLinear.from_bytes(raw, GpuQuantType.Q8_0, N, K, bias=bias.cuda())
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    cos, sin = rope_tables(D, max(mod, 8))
    cols = (2 * N // 3) // D * D
    # output rows N wide inside a buffer 16 columns wider (row stride N + 16), at column 8
    buf = torch.full((M, N + 16), 7.0, dtype=torch.bfloat16, device="cuda")
    rope = RopeEpilogue(rope_pair_table(torch.from_numpy(cos), torch.from_numpy(sin)).cuda(),
                        cols, D, off, div, mod)
    lin.forward(x.cuda(), out=buf[:, 8:8 + N], rope=rope)
    torch.cuda.synchronize()
    b = to_np(buf)
    assert np.all(b[:, :8] == 7.0) and np.all(b[:, 8 + N:] == 7.0)  # nothing outside the slice
    rows = slice(0, min(M, 256))
    mm = oracle.q8_0_matmul(np.frombuffer(raw, np.uint8), N, K, to_np(x[rows])) + to_np(bias)
    ref = _rope_ref(mm, cos, sin, cols, D, off, div, mod)
    assert rel_err(b[rows, 8:8 + N], ref) < TOL_HALF
    if M > 256:  # the last rows' positions
        mm = oracle.q8_0_matmul(np.frombuffer(raw, np.uint8), N, K, to_np(x[-64:])) + to_np(bias)
        ref = _rope_ref(mm, cos, sin, cols, D, off + M - 64, div, mod)
        assert rel_err(b[-64:, 8:8 + N], ref) < TOL_HALF


def test_fp8_linear_rope_epilogue():
    from sketchpad_b200.flux import rope_tables
    from sketchpad_b200.quantized_matmul import RopeEpilogue, rope_pair_table
    M, N, K, D = 512, 3 * 640, 640, 128
    g = torch.Generator(device="cpu").manual_seed(9)
    w = torch.randn(N, K, generator=g) * 0.02
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    lin = Fp8Linear.from_weight(w.cuda(), bias.cuda(), Fp8Config.e4m3().with_per_channel(True))
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    cos, sin = rope_tables(D, 100)
    rope = RopeEpilogue(rope_pair_table(torch.from_numpy(cos), torch.from_numpy(sin)).cuda(),
                        2 * 640, D, 0, 1, 100)
    y = lin.forward(x.cuda(), rope=rope)
    # the same product written as f16 (the attention-input dtype of the Wan harness)
    y16 = lin.forward(x.cuda(), rope=rope, out_dtype=torch.float16)
    torch.cuda.synchronize()
    assert y16.dtype == torch.float16
    wdq = to_np(lin.weight.dequantize())
    rows = slice(0, 256)
    ref = _rope_ref(oracle.linear_nt(to_np(x[rows]), wdq, to_np(bias)), cos, sin, 2 * 640, D,
                    0, 1, 100)
    assert rel_err(to_np(y[rows]), ref) < TOL_HALF
    # f16's rounding is 8x finer than bf16's: the error shrinks accordingly
    e16 = rel_err(to_np(y16[rows]), ref)
    assert e16 < 2e-3 and e16 < rel_err(to_np(y[rows]), ref)


def test_rope_epilogue_rejects_bad_geometry():
    from sketchpad_b200.quantized_matmul import RopeEpilogue
    lin = GpuQuantizedLinear.from_bytes(make_q8_0_synthetic(64, 64, seed=1), GpuQuantType.Q8_0,
                                        64, 64)
    x = torch.randn(8, 64, device="cuda").to(torch.bfloat16)
    tab = torch.zeros(4, 8, 2, device="cuda")
    with pytest.raises(Exception, match="positions"):
        lin.forward(x, rope=RopeEpilogue(tab, 32, 16, 0, 1, 5))  # mod > table rows
    with pytest.raises(Exception, match="head_dim"):
        lin.forward(x, rope=RopeEpilogue(tab, 36, 12, 0, 1, 4))  # 8 does not divide 12


_KQ_CASES = [("Q4K", 12), ("Q2K", 10), ("Q3K", 11)]


@pytest.mark.parametrize("name,fmt", _KQ_CASES)
@pytest.mark.parametrize("N,K", [(64, 512), (300, 1024)])
def test_kquant_dequant_bit_exact(name, fmt, N, K):
    from sketchpad_b200.quantized_matmul import make_kquant_synthetic
    qt = GpuQuantType[name]
    raw = make_kquant_synthetic(qt, N, K, seed=fmt + N)
    lin = GpuQuantizedLinear.from_bytes(raw, qt, N, K)
    got = to_np(lin.dequantize())
    ref = oracle.kquant_dequantize(fmt, np.frombuffer(raw, np.uint8), N * K).reshape(N, K)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("name,fmt", _KQ_CASES)
@pytest.mark.parametrize("M,N,K", [(200, 256, 512), (4608, 3072, 3072), (77, 48, 256)])
def test_kquant_linear_vs_oracle(name, fmt, M, N, K):
    from sketchpad_b200.quantized_matmul import make_kquant_synthetic
    qt = GpuQuantType[name]
    raw = make_kquant_synthetic(qt, N, K, seed=M + fmt)
    g = torch.Generator(device="cpu").manual_seed(M)
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    lin = GpuQuantizedLinear.from_bytes(raw, qt, N, K, bias=bias.cuda())
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    y = lin.forward(x.cuda())
    torch.cuda.synchronize()
    w = oracle.kquant_dequantize(fmt, np.frombuffer(raw, np.uint8), N * K).reshape(N, K)
    rows = slice(0, min(M, 256))
    ref = oracle.linear_nt(to_np(x[rows]), w, to_np(bias))
    assert rel_err(to_np(y[rows]), ref) < TOL_HALF
    if M > 256:
        ref_tail = oracle.linear_nt(to_np(x[-64:]), w, to_np(bias))
        assert rel_err(to_np(y[-64:]), ref_tail) < TOL_HALF


def test_kquant_linear_rejects_bad_shapes():
    from sketchpad_b200 import _lib
    from sketchpad_b200.quantized_matmul import make_kquant_synthetic
    lin = GpuQuantizedLinear.from_bytes(make_kquant_synthetic(GpuQuantType.Q4K, 16, 256),
                                        GpuQuantType.Q4K, 16, 256)
    with pytest.raises(ValueError, match="epilogue"):
        lin.forward(torch.zeros(4, 256, device="cuda", dtype=torch.bfloat16),
                    gate=torch.ones(16, device="cuda", dtype=torch.bfloat16))
    x = torch.zeros(4, 192, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(_lib.SketchpadError, match="multiple of 256"):
        _lib.call("sp_kquant_linear", 12, x.data_ptr(), lin.q.data_ptr(), lin.scale.data_ptr(),
                  lin.kmin.data_ptr(), None, x.data_ptr(), 4, 16, 192, _lib.SP_BF16, None)


@pytest.mark.parametrize("M,N,K", [(1, 18432, 3072), (512, 3072, 12288), (3, 9216, 3072)])
def test_splitk_small_grid_linear_vs_oracle(M, N, K):
    # the DiT modulation (M = 1) and text-stream (M = 512) GEMMs: tile grids of 24-72 CTAs,
    # run as split-K with the deterministic reduce; two calls give identical bytes
    raw = make_q8_0_synthetic(N, K, seed=N + M)
    g = torch.Generator(device="cpu").manual_seed(M + 1)
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    lin = GpuQuantizedLinear.from_bytes(raw, GpuQuantType.Q8_0, N, K, bias=bias.cuda())
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    y1, y2 = lin.forward(x), lin.forward(x)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    rows = slice(0, min(M, 64))
    ref = oracle.q8_0_matmul(np.frombuffer(raw, np.uint8), N, K, to_np(x[rows])) + to_np(bias)
    assert rel_err(to_np(y1[rows]), ref) < TOL_HALF



@pytest.mark.parametrize("kind", ["swiglu", "geglu"])
@pytest.mark.parametrize("M,F,K", [(200, 128, 256), (4096, 1536, 3072), (77, 640, 2048)])
def test_q8_0_linear_glu_epilogue(kind, M, F, K):
    # gate/up (value/gate) rows interleaved; y = silu(lo) * hi or lo * gelu(hi) from the f32
    # accumulators (glu.rs:91-96, blocks.rs:446-458); (77, 640, 2048) runs split-K
    from sketchpad_b200.quantized_matmul import GLU_GEGLU, GLU_SWIGLU, interleave_rows
    raw_a, raw_b = make_q8_0_synthetic(F, K, seed=F + 1), make_q8_0_synthetic(F, K, seed=F + 2)
    g = torch.Generator(device="cpu").manual_seed(M)
    ba = (torch.randn(F, generator=g) * 0.1).to(torch.bfloat16)
    bb = (torch.randn(F, generator=g) * 0.1).to(torch.bfloat16)
    la = GpuQuantizedLinear.from_bytes(raw_a, GpuQuantType.Q8_0, F, K)
    lb = GpuQuantizedLinear.from_bytes(raw_b, GpuQuantType.Q8_0, F, K)
    lin = GpuQuantizedLinear(interleave_rows(la.q, lb.q), interleave_rows(la.scale, lb.scale, dim=1),
                             2 * F, K, torch.bfloat16, interleave_rows(ba, bb).cuda())
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    y = lin.forward(x.cuda(), glu=GLU_SWIGLU if kind == "swiglu" else GLU_GEGLU)
    torch.cuda.synchronize()
    assert y.shape == (M, F)
    rows = slice(0, min(M, 128))
    lo = oracle.q8_0_matmul(np.frombuffer(raw_a, np.uint8), F, K, to_np(x[rows])) + to_np(ba)
    hi = oracle.q8_0_matmul(np.frombuffer(raw_b, np.uint8), F, K, to_np(x[rows])) + to_np(bb)
    ref = (oracle.activation(lo, "silu") * hi if kind == "swiglu"
           else lo * oracle.activation(hi, "gelu"))
    assert rel_err(to_np(y[rows]), ref) < TOL_HALF


def test_fp8_linear_glu_epilogue():
    from sketchpad_b200.quantized_matmul import GLU_SWIGLU, interleave_rows
    M, F, K = 300, 640, 640
    g = torch.Generator(device="cpu").manual_seed(4)
    wa, wb = torch.randn(F, K, generator=g) * 0.02, torch.randn(F, K, generator=g) * 0.02
    la = Fp8Linear.from_weight(wa.cuda(), None, Fp8Config.e4m3().with_per_channel(True))
    lb = Fp8Linear.from_weight(wb.cuda(), None, Fp8Config.e4m3().with_per_channel(True))
    lin = Fp8Linear(Fp8Tensor(interleave_rows(la.weight.data, lb.weight.data),
                              interleave_rows(la.weight.scale, lb.weight.scale),
                              Fp8Format.E4M3, (2 * F, K)), None)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    y = lin.forward(x.cuda(), glu=GLU_SWIGLU)
    torch.cuda.synchronize()
    rows = slice(0, 128)
    lo = oracle.linear_nt(to_np(x[rows]), to_np(la.weight.dequantize()))
    hi = oracle.linear_nt(to_np(x[rows]), to_np(lb.weight.dequantize()))
    assert rel_err(to_np(y[rows]), oracle.activation(lo, "silu") * hi) < TOL_HALF


@pytest.mark.parametrize("fmt", ["Q8_0", "FP8", "Q4K", "Q2K", "Q3K"])
@pytest.mark.parametrize("M,N,K", [(600, 272, 512), (1024, 768, 512), (300, 160, 256)])
def test_paired_tiles_bit_identical_to_unpaired(fmt, M, N, K):
    # sp_quant_linear_set_pairing(1): two-CTA clusters per 512 x 256 tile (cta_group::2 MMA);
    # ragged M (a peer CTA past the last row) and N (a peer's weight rows past N) included;
    # the f32 accumulation order per output is unchanged, so the bytes must match
    from sketchpad_b200.quantized_matmul import (make_kquant_synthetic, set_tile_pairing)
    g = torch.Generator(device="cpu").manual_seed(M + N)
    bias = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16).cuda()
    if fmt == "FP8":
        w = torch.randn(N, K, generator=g) * 0.02
        lin = Fp8Linear.from_weight(w.cuda(), bias, Fp8Config.e4m3().with_per_channel(True))
    elif fmt == "Q8_0":
        lin = GpuQuantizedLinear.from_bytes(make_q8_0_synthetic(N, K, seed=M), GpuQuantType.Q8_0,
                                            N, K, bias=bias)
    else:
        qt = GpuQuantType[fmt]
        lin = GpuQuantizedLinear.from_bytes(make_kquant_synthetic(qt, N, K, seed=M), qt, N, K,
                                            bias=bias)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    old = set_tile_pairing(False)
    try:
        y0 = lin.forward(x)
        set_tile_pairing(True)
        y1 = lin.forward(x)
        torch.cuda.synchronize()
    finally:
        set_tile_pairing(old)
    assert torch.equal(y0, y1)


