"""Shared helpers for the parity tests.

Error metric used throughout (and written next to every tolerance):
    rel_err(got, ref) = max|got - ref| / max|ref|
i.e. the max absolute deviation normalised by the reference's largest magnitude.  The bars
are the ones the build targets: 1e-3 for fp32-accumulate outputs, 2e-2 for bf16/f16
activations, exact equality for integer/byte work (dequantized weights).
"""
import numpy as np

TOL_F32 = 1e-3
TOL_HALF = 2e-2


def rel_err(got, ref) -> float:
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = np.abs(ref).max()
    return float(np.abs(got - ref).max() / (denom if denom > 0 else 1.0))


def to_np(t):
    return t.detach().float().cpu().numpy()
