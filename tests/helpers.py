"""Shared helpers for the parity tests.

Error metrics (written next to every tolerance):
    rel_err(got, ref)      = max|got - ref| / max|ref|
        the max absolute deviation normalised by the reference's largest magnitude: the bar
        every test asserts (1e-3 for fp32-accumulate outputs, 2e-2 for bf16/f16 activations,
        exact equality for integer/byte work such as dequantized weights);
    max_rel_err(got, ref)  = max_i |got_i - ref_i| / max(|ref_i|, floor),
        floor = ELEM_FLOOR * max|ref|
        the element-wise max relative error; elements far below the tensor's own scale are
        judged against the floor instead of their own (near-zero) magnitude.  Every rel_err
        call also records it, and the session summary prints both per test; tests that hold
        it to a bar say so.
"""
import os

import numpy as np

TOL_F32 = 1e-3
TOL_HALF = 2e-2
ELEM_FLOOR = 1e-2

# (test id, rel_err, max_rel_err) of every rel_err call in this session
PARITY_LOG = []


def max_rel_err(got, ref, floor_frac: float = ELEM_FLOOR) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    scale = np.abs(ref).max()
    floor = floor_frac * (scale if scale > 0 else 1.0)
    return float((np.abs(got - ref) / np.maximum(np.abs(ref), floor)).max())


def rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = np.abs(ref).max()
    e = float(np.abs(got - ref).max() / (denom if denom > 0 else 1.0))
    test = os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0]
    PARITY_LOG.append((test, e, max_rel_err(got, ref)))
    return e


def to_np(t):
    return t.detach().float().cpu().numpy()


def q8_linear_f32(lin):
    """(W [N, K] f32, bias [N] f32 or None) of a GpuQuantizedLinear, decoded by the oracle
    from GGUF Q8_0 blocks rebuilt out of the planar q / k-block-major scales."""
    import oracle
    q = lin.q.detach().cpu().numpy().astype(np.int8)
    s = lin.scale.detach().cpu().numpy().view(np.uint16)  # [K/32, N]
    N, K = q.shape
    blocks = np.empty((N, K // 32, 34), np.uint8)
    blocks[..., :2] = np.ascontiguousarray(s.T).view(np.uint8).reshape(N, K // 32, 2)
    blocks[..., 2:] = q.view(np.uint8).reshape(N, K // 32, 32)
    w = oracle.q8_0_dequantize(blocks.reshape(-1), N * K).reshape(N, K)
    b = None if lin.bias is None else to_np(lin.bias)
    return w, b


def fp8_linear_f32(lin):
    """(W [N, K] f32, bias or None) of an Fp8Linear: e4m3 bytes decoded by the oracle, times
    the per-channel (or per-tensor) scale as Fp8Tensor::dequantize does."""
    import oracle
    vals = oracle.e4m3_bytes_to_f32(lin.weight.data.detach().cpu().numpy())
    w = oracle.fp8_dequantize(vals, to_np(lin.weight.scale))
    b = None if lin.bias is None else to_np(lin.bias)
    return w, b


def split_rows(wb, i):
    """Split a stacked (W, b) pair at output row i (gate/up share one GEMM in the harness)."""
    w, b = wb
    return (w[:i], None if b is None else b[:i]), (w[i:], None if b is None else b[i:])


def split_interleaved(wb):
    """Split a row-interleaved (W, b) pair (first-half row j at 2j, second-half row j at
    2j+1: the GLU-epilogue layout) into its two halves."""
    w, b = wb
    return (w[0::2], None if b is None else b[0::2]), (w[1::2], None if b is None else b[1::2])
