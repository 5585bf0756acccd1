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
