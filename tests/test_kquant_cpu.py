"""K-quant weights (Q4_K, Q2_K, Q3_K) on the CPU: the oracle's restatement of the reference
decode (crates/sketchpad-convert/src/gguf.rs:737-871) against the reference's own golden
vector and hand-computed answers of its formulas, and the product library's lossless host
repack (decoded here with numpy f32 arithmetic) against the oracle, bit for bit."""
import numpy as np
import pytest

import oracle
from sketchpad_b200.quantized_matmul import (GpuQuantType, make_kquant_synthetic,
                                             repack_kquant_host)

F16_ONE, F16_HALF, F16_TWO = 0x3C00, 0x3800, 0x4000


def _put16(blk, off, bits):
    blk[off], blk[off + 1] = bits & 0xFF, bits >> 8


def test_q4_k_zero_block_golden():
    # gguf.rs:5455-5462: an all-zero Q4_K block decodes to zeros
    out = oracle.kquant_dequantize(12, np.zeros(144, np.uint8), 256)
    assert np.all(np.abs(out) < 1e-6)


def test_q4_k_known_answers():
    blk = np.zeros(144, np.uint8)
    _put16(blk, 0, F16_ONE)    # d = 1
    _put16(blk, 2, F16_HALF)   # dmin = 0.5
    blk[4 + 0] = 0xC2          # sub-block 0 scale = 0xC2 & 63 = 2; its top bits feed scale 4
    blk[4 + 4] = 0x03          # sub-block 0 min = 3
    blk[4 + 8] = 0x71          # sub-block 4: scale low nibble 1, min low nibble 7
    blk[16 + 0] = 0x5A         # sub-block 0, values 0 (lo = 10) and 16 (hi = 5)
    blk[16 + 4 * 16] = 0x0F    # sub-block 4, value 128 (lo = 15), value 144 (hi = 0)
    out = oracle.kquant_dequantize(12, blk, 256)
    assert out[0] == 1 * 2 * 10 - 0.5 * 3        # 18.5
    assert out[16] == 1 * 2 * 5 - 0.5 * 3        # 8.5
    sc4, m4 = 1 | (0xC2 >> 6) << 4, 7 | (0x03 >> 6) << 4   # 49, 7
    assert out[128] == sc4 * 15 - 0.5 * m4
    assert out[144] == -0.5 * m4


def test_q2_k_known_answers():
    blk = np.zeros(84, np.uint8)
    blk[0] = 0x31                      # sub-block 0: scale 1, min 3
    blk[16] = 0xE4                     # values 0..3: q = 0, 1, 2, 3 (low bits first)
    _put16(blk, 80, F16_ONE)
    _put16(blk, 82, F16_HALF)
    out = oracle.kquant_dequantize(10, blk, 256)
    assert list(out[:4]) == [-1.5, -0.5, 0.5, 1.5]
    assert np.all(out[16:] == 0.0)     # scale 0, min 0 elsewhere


def test_q3_k_known_answers():
    blk = np.zeros(110, np.uint8)
    blk[0] = 0x01                      # hmask: value 0 has the high bit
    blk[32] = 0xE4                     # low 2 bits of values 0..3: 0, 1, 2, 3
    blk[96] = 33                       # 6-bit field 33 -> scale 1 for sub-block 0
    _put16(blk, 108, F16_TWO)          # d = 2
    out = oracle.kquant_dequantize(11, blk, 256)
    assert list(out[:4]) == [0.0, -6.0, -4.0, -2.0]   # 2 * 1 * ((low2 | h << 2) - 4)
    # sub-blocks 8..15 take bits 6..11 of the first 32-bit word: byte 0's top two bits and
    # byte 1's low nibble (gguf.rs:791-803): field 8 = (0x61 >> 6) | (0x0B & 0xF) << 2 = 45
    blk2 = blk.copy()
    blk2[96], blk2[97] = 0x61, 0x0B
    scale8 = ((0x61 >> 6) | ((0x0B & 0x0F) << 2)) - 32   # 13
    scale1 = (0x0B & 0x3F) - 32                          # -21
    out2 = oracle.kquant_dequantize(11, blk2, 256)
    assert out2[0] == 0.0 and out2[1] == -6.0            # sub-block 0 keeps scale 1
    assert out2[16] == 2.0 * scale1 * (0 - 4)            # value 16: q = 0
    assert out2[128] == 2.0 * scale8 * (0 - 4)


def _decode_repacked(qp, a, b, off, sub):
    n, khalf = qp.shape
    q = np.empty((n, 2 * khalf), np.float32)
    q[:, 0::2] = qp & 0x0F
    q[:, 1::2] = qp >> 4
    q -= np.float32(off)
    af = np.repeat(a.T, sub, axis=1)  # [n, K]
    bf = np.repeat(b.T, sub, axis=1)
    return (af * q).astype(np.float32) - bf


@pytest.mark.parametrize("qt,fmt,off,sub", [(GpuQuantType.Q4K, 12, 0, 32),
                                             (GpuQuantType.Q2K, 10, 0, 16),
                                             (GpuQuantType.Q3K, 11, 4, 16)])
@pytest.mark.parametrize("N,K", [(3, 256), (40, 1024)])
def test_host_repack_is_lossless(qt, fmt, off, sub, N, K):
    raw = make_kquant_synthetic(qt, N, K, seed=N + K)
    qp, a, b = repack_kquant_host(raw, qt, N, K)
    got = _decode_repacked(qp, a, b, off, sub)
    ref = oracle.kquant_dequantize(fmt, np.frombuffer(raw, np.uint8), N * K).reshape(N, K)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_host_repack_rejects_bad_shapes():
    from sketchpad_b200 import _lib
    raw = make_kquant_synthetic(GpuQuantType.Q4K, 2, 256)
    with pytest.raises(_lib.SketchpadError, match="multiple of 256"):
        repack_kquant_host(raw, GpuQuantType.Q4K, 2, 128)
    with pytest.raises(_lib.SketchpadError, match="bytes"):
        repack_kquant_host(raw[:100], GpuQuantType.Q4K, 2, 256)
