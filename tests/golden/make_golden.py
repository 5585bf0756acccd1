"""Generate the golden fixtures under tests/golden/ from the reference's own known-answer tests.

The reference (rhi-zone/sketchpad, pure Rust) cannot be built in this image (no cargo/rustc),
so its known-answer tests are restated here case by case: the inputs are rebuilt exactly as
each Rust test builds them and the expected values/tolerances are the ones that test asserts.
Where the reference's formula fixes the answer exactly, an independent pure-Python
restatement of that formula also records the exact value (``exact``), which pins the C++
oracle more tightly than the Rust test's tolerance does.

Run:  python tests/golden/make_golden.py     (rewrites tests/golden/*.json)
"""
from __future__ import annotations

import json
import math
import os
import struct

HERE = os.path.dirname(os.path.abspath(__file__))


def f16_bits(v: float) -> int:
    """IEEE binary16 round-to-nearest-even (the `half` crate's f16::from_f32)."""
    return struct.unpack("<H", struct.pack("<e", v))[0]


def f16_value(bits: int) -> float:
    return struct.unpack("<e", struct.pack("<H", bits))[0]


def ref_test_f32_to_f16_bytes(val: float) -> int:
    """crates/sketchpad-llm/src/quantized.rs:473-493 -- the test helper's own f16 encoder
    (truncating mantissa, flushes values below 2^-14 to zero)."""
    bits = struct.unpack("<I", struct.pack("<f", val))[0]
    sign = (bits >> 31) & 1
    exp = ((bits >> 23) & 0xFF) - 127
    frac = bits & 0x7FFFFF
    if exp > 15:
        h = (sign << 15) | 0x7C00
    elif exp < -14:
        h = sign << 15
    else:
        h = (sign << 15) | (((exp + 15) & 0x1F) << 10) | (frac >> 13)
    return h & 0xFFFF


def f32(v: float) -> float:
    return struct.unpack("<f", struct.pack("<f", v))[0]


def rust_round(v: float) -> float:
    """f32::round: half away from zero."""
    return math.copysign(math.floor(abs(v) + 0.5), v)


def fp8_scalar_py(value: float, fmt: int) -> float:
    """crates/sketchpad-core/src/quantization.rs:451-492 restated in Python (f32 steps)."""
    max_val = 448.0 if fmt == 0 else 57344.0
    min_sub = 2.0 ** -9 if fmt == 0 else 2.0 ** -16
    mant = 3 if fmt == 0 else 2
    if math.isnan(value):
        return float("nan")
    if math.isinf(value):
        return max_val if value > 0 else -max_val
    sign = -1.0 if math.copysign(1.0, value) < 0 else 1.0
    a = abs(value)
    if a > max_val:
        return sign * max_val
    if a < min_sub:
        return 0.0
    e = math.floor(math.log2(a))
    ms = 2.0 ** e
    normalized = f32(a / ms)
    steps = float(2 ** mant)
    qm = f32(rust_round(f32((normalized - 1.0) * steps)) / steps + 1.0)
    return f32(sign * qm * ms)


def make_q8_0_data_ref(weights):
    """crates/sketchpad-llm/src/quantized.rs:495-513 (make_q8_0_data) restated."""
    out = bytearray()
    for i in range(0, len(weights), 32):
        block = [f32(w) for w in weights[i:i + 32]]
        max_abs = max(abs(v) for v in block)
        scale = f32(max_abs / 127.0) if max_abs > 0 else 0.0
        out += struct.pack("<H", ref_test_f32_to_f16_bytes(scale))
        for v in block:
            if scale > 0:
                q = int(max(-128.0, min(127.0, rust_round(f32(v / scale)))))
            else:
                q = 0
            out += struct.pack("<b", q)
    return bytes(out)


def main():
    cases = {}

    # gguf.rs:5390-5412 test_dequantize_q8_0: scale 0.5 via f16, quants i-16, |err| < 1e-6
    sb = f16_bits(0.5)
    quants = [i - 16 for i in range(32)]
    block = struct.pack("<H", sb) + bytes((q & 0xFF) for q in quants)
    cases["q8_0_decode_scale_half"] = {
        "source": "crates/sketchpad-convert/src/gguf.rs:5390-5412",
        "bytes_hex": block.hex(),
        "n_elements": 32,
        "expected": [f16_value(sb) * q for q in quants],
        "tol": 1e-6,
        "exact": True,
    }

    # gguf.rs:5541-5562 test_dequantize_q8_0_known_values: scale 1.0, q = 1,-1,127,-128,0,...
    q2 = [0] * 32
    q2[0], q2[1], q2[2], q2[3] = 1, -1, 127, -128
    block2 = struct.pack("<H", f16_bits(1.0)) + bytes((q & 0xFF) for q in q2)
    cases["q8_0_decode_known_values"] = {
        "source": "crates/sketchpad-convert/src/gguf.rs:5541-5562",
        "bytes_hex": block2.hex(),
        "n_elements": 32,
        "expected": [float(q) for q in q2],
        "check_first": 5,
        "tol": 1e-3,
        "exact": True,
    }

    # quantized.rs:516-552 test_quantized_tensor_matmul: 2x32 weights, input ones at 0,1
    row0 = [0.0] * 32
    row1 = [0.0] * 32
    row0[0], row0[1], row1[0], row1[1] = 1.0, 2.0, 3.0, 4.0
    data = make_q8_0_data_ref(row0 + row1)
    x = [0.0] * 32
    x[0] = x[1] = 1.0
    cases["q8_0_matmul_2x32"] = {
        "source": "crates/sketchpad-llm/src/quantized.rs:516-552",
        "bytes_hex": data.hex(),
        "out_features": 2,
        "in_features": 32,
        "input": x,
        "n_tokens": 1,
        "expected": [3.0, 7.0],
        "tol": 0.1,
    }

    # quantization.rs:793-812 test_quantize_fp8_scalar (E4M3)
    scal = []
    for v, exp_v, tol in [(1.5, 1.5, 0.01), (1.234, 1.25, 0.1), (1000.0, 448.0, 1.0),
                          (0.0, 0.0, 0.0), (-2.0, -2.0, 0.1)]:
        scal.append({"input": v, "expected": exp_v, "tol": tol,
                     "exact": fp8_scalar_py(f32(v), 0)})
    cases["fp8_e4m3_scalar"] = {
        "source": "crates/sketchpad-core/src/quantization.rs:793-812",
        "format": 0,
        "cases": scal,
    }

    # Formula-exact grid points of quantize_fp8_scalar (E4M3 and E5M2), including the
    # round-half-away ties and the sub-2^-6 region where the simulated grid keeps 3
    # mantissa bits (quantization.rs:451-492).
    grid_inputs = [1.0625, 1.1875, -1.0625, 0.3, 3.14159, 447.0, 449.0, 240.0, 232.0,
                   2.0 ** -6, 1.0625 * 2.0 ** -8, 0.001953125, 0.0019, 1e-4, 6e-3, 17.0,
                   -300.0, 57000.0, 60000.0, 0.07, 5000.0]
    cases["fp8_formula_grid"] = {
        "source": "crates/sketchpad-core/src/quantization.rs:451-492",
        "cases": [{"input": v, "format": fmt, "exact": fp8_scalar_py(f32(v), fmt)}
                  for fmt in (0, 1) for v in grid_inputs],
    }

    # quantization.rs:815-831 test_quantize_fp8_tensor (per-tensor, max diff < 0.5)
    cases["fp8_tensor_per_tensor"] = {
        "source": "crates/sketchpad-core/src/quantization.rs:815-831",
        "input": [[1.0, 2.0, 3.0, 4.0], [0.5, 1.5, 2.5, 3.5]],
        "per_channel": False, "format": 0, "max_diff": 0.5, "n_scales": 1,
    }
    # quantization.rs:834-848 test_quantize_fp8_per_channel (scale dims == rows, diff < 5)
    cases["fp8_tensor_per_channel"] = {
        "source": "crates/sketchpad-core/src/quantization.rs:834-848",
        "input": [[1.0, 2.0], [100.0, 200.0]],
        "per_channel": True, "format": 0, "max_diff": 5.0, "n_scales": 2,
    }
    # quantization.rs:883-898 test_fp8_e5m2 (diff < 200)
    cases["fp8_e5m2_tensor"] = {
        "source": "crates/sketchpad-core/src/quantization.rs:883-898",
        "input": [[100.0, 500.0, 1000.0, 5000.0]],
        "per_channel": False, "format": 1, "max_diff": 200.0, "n_scales": 1,
    }
    # quantization.rs:851-870 test_fp8_linear (shape [1,3])
    cases["fp8_linear_shape"] = {
        "source": "crates/sketchpad-core/src/quantization.rs:851-870",
        "weight": [[1.0, 2.0, 3.0, 4.0], [0.1, 0.2, 0.3, 0.4], [-1.0, -2.0, -3.0, -4.0]],
        "input": [[1.0, 1.0, 1.0, 1.0]],
        "out_shape": [1, 3],
    }

    # Hand-computed answers of the GroupNorm formula (groupnorm.rs:62-102): one group of
    # [1,2,3,4]: mean 2.5, biased var 1.25.
    gn_x = [1.0, 2.0, 3.0, 4.0]
    den = math.sqrt(1.25 + 1e-5)
    gn_norm = [(v - 2.5) / den for v in gn_x]
    cases["groupnorm_known_answer"] = {
        "source": "crates/sketchpad-core/src/groupnorm.rs:62-102 (hand-computed)",
        "shape": [1, 2, 1, 2], "groups": 1, "eps": 1e-5,
        "input": gn_x, "gamma": [2.0, 0.5], "beta": [0.25, -1.0],
        "expected_norm": [gn_norm[0] * 2 + 0.25, gn_norm[1] * 2 + 0.25,
                          gn_norm[2] * 0.5 - 1.0, gn_norm[3] * 0.5 - 1.0],
        "tol": 1e-6,
    }
    # Attention known answer (blocks.rs:393-401): equal scores -> mean of V rows; one
    # dominant key -> that key's V row.
    cases["attention_known_answer"] = {
        "source": "crates/sketchpad-unet/src/blocks.rs:393-401 (hand-computed)",
        "q": [[0.0, 0.0]], "k": [[1.0, 2.0], [3.0, -1.0], [0.5, 0.5]],
        "v": [[1.0, 10.0], [2.0, 20.0], [6.0, 0.0]],
        "expected": [[3.0, 10.0]],
        "tol": 1e-6,
    }

    for name, case in cases.items():
        with open(os.path.join(HERE, name + ".json"), "w") as fh:
            json.dump(case, fh, indent=1)
    print(f"wrote {len(cases)} fixtures to {HERE}")


if __name__ == "__main__":
    main()
