"""Weight-file readers (sp_model_*, sketchpad_b200/loaders.py) on synthetic files written here.

GGUF v3 as crates/sketchpad-convert/src/gguf.rs:351-470 reads it (little-endian header,
typed metadata values incl. nested arrays, tensor infos with innermost-first dimensions,
data at the header end rounded up to 32 bytes); safetensors as the `safetensors` crate that
crates/sketchpad-convert/src/loader.rs uses lays it out (u64 header length, JSON header,
data_offsets relative to the data section).  CPU: parsing, bytes, conversions, errors, and
the Q8_0 / K-quant repack of loaded bytes; GPU: the loaded layers' forward vs the oracle.
"""
import json
import struct

import numpy as np
import pytest
import torch

import oracle
from helpers import TOL_HALF, rel_err, to_np
from sketchpad_b200 import loaders as LD
from sketchpad_b200.quantized_matmul import make_kquant_synthetic, make_q8_0_synthetic, GpuQuantType


def _gguf_str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path, tensors, metadata=(), version=3, truncate=0, bad_offset=False):
    """tensors: [(name, ggml_type, row-major shape, raw bytes)]."""
    out = struct.pack("<IIQQ", 0x46554747, version, len(tensors), len(metadata))
    for key, vtype, payload in metadata:
        out += _gguf_str(key) + struct.pack("<I", vtype) + payload
    offs, data = [], b""
    for name, t, shape, raw in tensors:
        data += b"\0" * ((-len(data)) % 32)
        offs.append(len(data))
        data += raw
    for (name, t, shape, raw), off in zip(tensors, offs):
        dims = list(reversed(shape))  # innermost first on disk
        out += _gguf_str(name) + struct.pack("<I", len(dims))
        out += b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", t, off + (1 << 30 if bad_offset else 0))
    out += b"\0" * ((-len(out)) % 32)
    blob = out + data
    open(path, "wb").write(blob[:len(blob) - truncate] if truncate else blob)


META = [("general.architecture", 8, _gguf_str("flux")),
        ("general.alignment", 4, struct.pack("<I", 32)),
        ("tokenizer.tokens", 9, struct.pack("<IQ", 8, 2) + _gguf_str("a") + _gguf_str("bc")),
        ("nested", 9, struct.pack("<IQ", 9, 1) + struct.pack("<IQ", 6, 2) +
         struct.pack("<ff", 1.0, 2.0)),
        ("scale", 6, struct.pack("<f", 0.5))]


def _gguf_fixture(tmp_path):
    q8 = make_q8_0_synthetic(64, 128, seed=3)
    q4 = make_kquant_synthetic(GpuQuantType.Q4K, 16, 256, seed=4)
    f32 = np.arange(15, dtype=np.float32).reshape(3, 5) * 0.25
    f16 = np.linspace(-2, 2, 7).astype(np.float16)
    path = tmp_path / "m.gguf"
    write_gguf(path, [("blk.0.w", 8, (64, 128), q8), ("blk.0.k", 12, (16, 256), q4),
                      ("norm", 0, (3, 5), f32.tobytes()), ("b16", 1, (7,), f16.tobytes())], META)
    return path, q8, q4, f32, f16


def test_gguf_reader_tensors_metadata_and_bytes(tmp_path):
    path, q8, q4, f32, f16 = _gguf_fixture(tmp_path)
    with LD.ModelFile(str(path)) as f:
        assert f.container == LD.CONTAINER_GGUF
        assert f.metadata_keys == [k for k, _, _ in META]
        w = f.info("blk.0.w")
        assert (w.ggml_type, w.shape, w.nbytes) == (8, (64, 128), 64 * 4 * 34)
        assert f.info("blk.0.k").shape == (16, 256) and f.info("blk.0.k").ggml_type == 12
        assert bytes(f.raw("blk.0.w")) == q8 and bytes(f.raw("blk.0.k")) == q4
        assert np.array_equal(f.load_f32("norm").numpy(), f32)
        assert np.array_equal(f.load_f32("b16").numpy(), f16.astype(np.float32))
        # the loaded Q8_0 bytes decode exactly as the reference's CPU path (oracle)
        ref = oracle.q8_0_dequantize(np.frombuffer(q8, np.uint8), 64 * 128)
        assert np.array_equal(oracle.q8_0_dequantize(f.raw("blk.0.w"), 64 * 128), ref)
        # and repack into the planar layout the fused GEMM reads (host side, no GPU)
        lin = f.quantized_linear("blk.0.w", device="cpu")
        assert lin.q.shape == (64, 128) and lin.out_features == 64 and lin.in_features == 128
        klin = f.quantized_linear("blk.0.k", device="cpu")
        assert klin.quant_type == GpuQuantType.Q4K
        with pytest.raises(TypeError):
            f.quantized_linear("norm", device="cpu")
        with pytest.raises(KeyError):
            f.info("missing")


@pytest.mark.parametrize("kind", ["magic", "version", "truncated", "offset", "type"])
def test_gguf_reader_rejects_malformed_files(tmp_path, kind):
    path = tmp_path / "bad.gguf"
    q8 = make_q8_0_synthetic(32, 64, seed=5)
    if kind == "magic":
        path.write_bytes(b"GGUX" + b"\0" * 60)
    elif kind == "version":
        write_gguf(path, [("w", 8, (32, 64), q8)], version=2)
    elif kind == "truncated":
        write_gguf(path, [("w", 8, (32, 64), q8)], truncate=100)
    elif kind == "offset":
        write_gguf(path, [("w", 8, (32, 64), q8)], bad_offset=True)
    else:
        write_gguf(path, [("w", 99, (32, 64), q8)])
    with pytest.raises(Exception) as e:
        LD.ModelFile(str(path))
    assert "sp_model_open" in str(e.value) or "GGUF" in str(e.value)


def write_safetensors(path, tensors, metadata=None, corrupt=False):
    """tensors: [(name, dtype string, shape, raw bytes)]."""
    header, data = {}, b""
    for name, dt, shape, raw in tensors:
        header[name] = {"dtype": dt, "shape": list(shape),
                        "data_offsets": [len(data), len(data) + len(raw) + (8 if corrupt else 0)]}
        data += raw
    if metadata:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    h += b" " * ((-len(h)) % 8)
    open(path, "wb").write(struct.pack("<Q", len(h)) + h + data)


def _fp8_fixture(tmp_path, N=256, K=128):
    rng = np.random.default_rng(7)
    # random finite e4m3 codes (0x7F / 0xFF are NaN) and per-channel scales
    codes = rng.integers(0, 255, size=(N, K)).astype(np.uint8)
    codes[(codes & 0x7F) == 0x7F] ^= 1
    data = oracle.e4m3_bytes_to_f32(codes).reshape(N, K)
    scale = rng.uniform(1e-4, 1e-3, N).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    b16 = (torch.from_numpy(bias).to(torch.bfloat16).view(torch.int16).numpy()).tobytes()
    path = tmp_path / "w.safetensors"
    write_safetensors(path, [("layer.weight", "F8_E4M3", (N, K), codes.tobytes()),
                             ("layer.weight_scale", "F32", (N,), scale.astype(np.float32).tobytes()),
                             ("layer.bias", "BF16", (N,), b16)],
                      metadata={"format": "pt"})
    return path, data, scale, codes, bias


def test_safetensors_reader_fp8_weights(tmp_path):
    path, data, scale, codes, bias = _fp8_fixture(tmp_path)
    with LD.ModelFile(str(path)) as f:
        assert f.container == LD.CONTAINER_SAFETENSORS and f.metadata_keys == ["format"]
        info = f.info("layer.weight")
        assert info.type == LD.T_F8_E4M3 and info.shape == (256, 128) and info.nbytes == 256 * 128
        raw = f.raw("layer.weight")
        assert np.array_equal(raw, codes.reshape(-1))
        # e4m3 bytes decode to exactly the reference's rounded values
        assert np.array_equal(oracle.e4m3_bytes_to_f32(np.array(raw)).reshape(256, 128), data)
        assert np.array_equal(f.load_f32("layer.weight_scale").numpy(), scale)
        b = f.load_f32("layer.bias").numpy()
        assert np.array_equal(b, torch.from_numpy(bias).to(torch.bfloat16).float().numpy())


@pytest.mark.parametrize("kind", ["offsets", "dtype", "header"])
def test_safetensors_reader_rejects_malformed_files(tmp_path, kind):
    path = tmp_path / "bad.safetensors"
    raw = np.zeros(8, np.float32).tobytes()
    if kind == "offsets":
        write_safetensors(path, [("x", "F32", (8,), raw)], corrupt=True)
    elif kind == "dtype":
        write_safetensors(path, [("x", "F4", (8,), raw)])
    else:
        path.write_bytes(struct.pack("<Q", 12) + b'{"x": [1, 2' + b"\0")
    with pytest.raises(Exception):
        LD.ModelFile(str(path))


@pytest.mark.gpu
def test_loaded_layers_forward_vs_oracle(tmp_path):
    gpath, q8, _, _, _ = _gguf_fixture(tmp_path)
    x = torch.randn(96, 128, generator=torch.Generator().manual_seed(8)).to(torch.bfloat16)
    with LD.ModelFile(str(gpath)) as f:
        lin = f.quantized_linear("blk.0.w")
        y = lin.forward(x.cuda())
    ref = oracle.q8_0_matmul(np.frombuffer(q8, np.uint8), 64, 128, to_np(x))
    assert rel_err(to_np(y), ref) < TOL_HALF
    spath, data, scale, _, bias = _fp8_fixture(tmp_path)
    with LD.ModelFile(str(spath)) as f:
        fl = f.fp8_linear("layer.weight", scale="layer.weight_scale", bias="layer.bias")
        yf = fl.forward(x.cuda())
    b16 = torch.from_numpy(bias).to(torch.bfloat16).float().numpy()
    ref = oracle.linear_nt(to_np(x), oracle.fp8_dequantize(data, scale), b16)
    assert rel_err(to_np(yf), ref) < TOL_HALF
