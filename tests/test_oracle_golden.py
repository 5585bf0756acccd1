"""Pin the CPU oracle to the reference's own known-answer tests (tests/golden/*.json).

Each fixture restates one Rust test of rhi-zone/sketchpad (its `source` field gives the
file:line); make_golden.py documents how the inputs were rebuilt.
"""
import json
import math
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    with open(os.path.join(GOLD, name + ".json")) as fh:
        return json.load(fh)


@pytest.mark.parametrize("name", ["q8_0_decode_scale_half", "q8_0_decode_known_values"])
def test_q8_0_decode_golden(name):
    case = load(name)
    data = np.frombuffer(bytes.fromhex(case["bytes_hex"]), np.uint8)
    out = oracle.q8_0_dequantize(data, case["n_elements"])
    exp = np.array(case["expected"], np.float32)
    n = case.get("check_first", len(exp))
    assert np.all(np.abs(out[:n] - exp[:n]) < case["tol"])
    if case.get("exact"):
        assert np.array_equal(out, exp)  # f16 scale * int8 is exact in f32


def test_q8_0_matmul_golden():
    case = load("q8_0_matmul_2x32")
    data = np.frombuffer(bytes.fromhex(case["bytes_hex"]), np.uint8)
    x = np.array(case["input"], np.float32).reshape(case["n_tokens"], case["in_features"])
    y = oracle.q8_0_matmul(data, case["out_features"], case["in_features"], x)
    assert np.all(np.abs(y.ravel() - np.array(case["expected"])) < case["tol"])


def test_fp8_scalar_golden():
    case = load("fp8_e4m3_scalar")
    for c in case["cases"]:
        got = oracle.fp8_quantize_scalar(c["input"], case["format"])
        if c["tol"] == 0.0:
            assert got == c["expected"]
        else:
            assert abs(got - c["expected"]) < c["tol"]
        assert got == c["exact"], (c, got)


def test_fp8_formula_grid():
    for c in load("fp8_formula_grid")["cases"]:
        got = oracle.fp8_quantize_scalar(c["input"], c["format"])
        assert got == c["exact"], (c, got)


@pytest.mark.parametrize("name", ["fp8_tensor_per_tensor", "fp8_tensor_per_channel",
                                  "fp8_e5m2_tensor"])
def test_fp8_tensor_golden(name):
    case = load(name)
    w = np.array(case["input"], np.float32)
    data, scale = oracle.fp8_quantize(w, case["format"], case["per_channel"])
    assert scale.size == case["n_scales"]
    deq = oracle.fp8_dequantize(data, scale)
    assert np.abs(deq - w).max() < case["max_diff"]


def test_fp8_linear_shape_golden():
    case = load("fp8_linear_shape")
    w = np.array(case["weight"], np.float32)
    data, scale = oracle.fp8_quantize(w, 0, False)
    y = oracle.linear_nt(np.array(case["input"], np.float32), oracle.fp8_dequantize(data, scale))
    assert list(y.shape) == case["out_shape"]
    # and it is x @ W^T of the dequantized weight
    assert np.allclose(y, np.array(case["input"], np.float32) @ oracle.fp8_dequantize(data, scale).T)


def test_groupnorm_known_answer():
    case = load("groupnorm_known_answer")
    x = np.array(case["input"], np.float32).reshape(case["shape"])
    y = oracle.groupnorm_act(x, np.array(case["gamma"], np.float32),
                             np.array(case["beta"], np.float32), case["groups"], case["eps"],
                             silu=False)
    assert np.abs(y.ravel() - np.array(case["expected_norm"])).max() < case["tol"]
    ys = oracle.groupnorm_act(x, np.array(case["gamma"], np.float32),
                              np.array(case["beta"], np.float32), case["groups"], case["eps"],
                              silu=True)
    e = np.array(case["expected_norm"])
    assert np.abs(ys.ravel() - e / (1 + np.exp(-e))).max() < case["tol"]


def test_attention_known_answer():
    case = load("attention_known_answer")
    q = np.array(case["q"], np.float32)[None]
    k = np.array(case["k"], np.float32)[None]
    v = np.array(case["v"], np.float32)[None]
    for variant in (0, 1):
        o = oracle.attention(q, k, v, variant=variant)
        assert np.abs(o[0] - np.array(case["expected"])).max() < case["tol"]
    # one dominant key -> its V row
    k2 = k.copy()
    k2[0, 1] = [200.0, 200.0]
    o = oracle.attention(np.ones_like(q), k2, v)
    assert np.abs(o[0, 0] - v[0, 1]).max() < 1e-5


def test_groupnorm_clamps_and_biased_variance():
    # F6: inputs are clamped to +-65000 before the statistics, and the variance is biased.
    x = np.array([1e6, -1e6, 3.0, 5.0], np.float32).reshape(1, 1, 2, 2)
    y = oracle.groupnorm_act(x, np.ones(1, np.float32), np.zeros(1, np.float32), 1, 1e-5,
                             silu=False)
    xc = np.clip(x.astype(np.float64), -65000, 65000).ravel()
    exp = (xc - xc.mean()) / math.sqrt(xc.var() + 1e-5)
    assert np.allclose(y.ravel(), exp, rtol=1e-6, atol=1e-6)


def test_f16_decode_all_bit_patterns():
    bits = np.arange(65536, dtype=np.uint16)
    f = oracle.f16_bits_to_f32(bits)
    ref = bits.view(np.float16).astype(np.float32)
    ok = ~np.isnan(ref)
    assert np.array_equal(f.view(np.uint32)[ok], ref.view(np.uint32)[ok])
    assert np.all(np.isnan(f[~ok]))


@pytest.mark.parametrize("silu", [False, True])
def test_groupnorm_f16_dtype_path(silu):
    # groupnorm.rs:76-99 on an f16 tensor, restated with numpy float16 arithmetic (each f16
    # op computes in f32 and rounds to nearest even, as the half crate does): f32 stats,
    # normalise in f32, cast to f16, x * weight and + bias as f16 ops, clamp, then
    # silu(x) = x * sigmoid(x) with sigmoid evaluated in f32 and cast to f16
    rng = np.random.default_rng(21)
    x16 = (rng.standard_normal((2, 8, 3, 5)) * 3 + 0.5).astype(np.float16)
    g16 = (rng.standard_normal(8) * 0.1 + 1).astype(np.float16)
    b16 = (rng.standard_normal(8) * 0.1).astype(np.float16)
    xg = x16.astype(np.float64).reshape(2, 4, -1)
    mean = xg.mean(axis=2, keepdims=True).astype(np.float32)
    var = ((xg - mean) ** 2).mean(axis=2, keepdims=True).astype(np.float32)
    xn = ((xg.astype(np.float32) - mean) / np.sqrt(var + np.float32(1e-5))).astype(np.float16)
    xn = xn.reshape(2, 8, 3, 5)
    v = xn * g16[None, :, None, None] + b16[None, :, None, None]  # f16 ops, each rounded
    v = np.clip(v, -65000, 65000).astype(np.float16)
    if silu:
        sig = (1.0 / (1.0 + np.exp(-v.astype(np.float32)))).astype(np.float16)
        v = v * sig
    y = oracle.groupnorm_act(x16.astype(np.float32), g16.astype(np.float32),
                             b16.astype(np.float32), 4, 1e-5, silu=silu, dtype="f16")
    # every oracle value is an f16 value; allow one f16 ulp for f32 exp/sqrt rounding
    assert np.array_equal(y.astype(np.float16).astype(np.float32), y)
    ulp = np.spacing(np.abs(v).astype(np.float16)).astype(np.float32)
    assert np.all(np.abs(y - v.astype(np.float32)) <= ulp)
    # and it differs from the f32 path (the dtype round trips are real)
    y32 = oracle.groupnorm_act(x16.astype(np.float32), g16.astype(np.float32),
                               b16.astype(np.float32), 4, 1e-5, silu=silu)
    assert not np.array_equal(y, y32)
