"""Bf16Linear (sp_bf16_linear*): plain bf16 weights on the tcgen05 GEMM, the UNet's projection
and feed-forward shapes (crates/sketchpad-unet/src/blocks.rs:213-231, :292-305, :446-458),
vs the oracle's f32 product of the same bf16 values.

Metric: rel_err = max|gpu - oracle| / max|oracle| < 2e-2 (bf16 output)."""
import numpy as np
import pytest
import torch

import oracle
from helpers import TOL_HALF, rel_err, to_np
from sketchpad_b200.linear import Bf16Linear
from sketchpad_b200.quantized_matmul import GLU_GEGLU, GLU_SWIGLU

pytestmark = pytest.mark.gpu


def _bf(seed, *shape, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(8192, 960, 320), (2048, 640, 640), (512, 1280, 1280),
                                   (154, 640, 768), (2, 1280, 320), (300, 48, 64)])
def test_bf16_linear_vs_oracle(M, N, K):
    x, w, b = _bf(1, M, K), _bf(2, N, K, scale=0.02), _bf(3, N, scale=0.02)
    lin = Bf16Linear(w.cuda(), b.cuda())
    y = lin.forward(x.cuda())
    torch.cuda.synchronize()
    rows = np.r_[0:min(M, 256), max(0, M - 64):M]
    ref = oracle.linear_nt(to_np(x)[rows], to_np(w), to_np(b))
    assert rel_err(to_np(y)[rows], ref) < TOL_HALF


def test_bf16_linear_residual_accumulates_in_place():
    # the UNet transformer's `resid += x @ W` (no bias), written into resid by the epilogue
    M, N, K = 4096, 320, 1280
    x, w = _bf(4, M, K), _bf(5, N, K, scale=0.02)
    r = _bf(6, M, N)
    rg = r.cuda().clone()
    lin = Bf16Linear(w.cuda())
    out = lin.forward(x.cuda(), out=rg, residual=rg)
    torch.cuda.synchronize()
    assert out.data_ptr() == rg.data_ptr()
    rows = slice(0, 256)
    ref = to_np(r)[rows] + oracle.linear_nt(to_np(x)[rows], to_np(w), None)
    assert rel_err(to_np(rg)[rows], ref) < TOL_HALF


@pytest.mark.parametrize("kind", [GLU_GEGLU, GLU_SWIGLU])
def test_bf16_linear_glu_epilogue(kind):
    # GEGLU (blocks.rs:446-458: value * gelu(gate)) from row-interleaved weights
    M, F, K = 2048, 1280, 320
    x = _bf(7, M, K)
    wv, wg = _bf(8, F, K, scale=0.05), _bf(9, F, K, scale=0.05)
    bv, bg = _bf(10, F, scale=0.02), _bf(11, F, scale=0.02)
    lin = Bf16Linear.glu(Bf16Linear(wv.cuda(), bv.cuda()), Bf16Linear(wg.cuda(), bg.cuda()))
    y = lin.forward(x.cuda(), glu=kind)
    torch.cuda.synchronize()
    assert y.shape == (M, F)
    rows = slice(0, 256)
    v = oracle.linear_nt(to_np(x)[rows], to_np(wv), to_np(bv))
    g = oracle.linear_nt(to_np(x)[rows], to_np(wg), to_np(bg))
    ref = v * oracle.activation(g, "gelu") if kind == GLU_GEGLU else oracle.activation(v, "silu") * g
    assert rel_err(to_np(y)[rows], ref) < TOL_HALF


def test_bf16_linear_rejects_bad_shapes():
    with pytest.raises(ValueError):
        Bf16Linear(torch.zeros(48, 100, dtype=torch.bfloat16, device="cuda"))
