"""LayerNorm (unbiased variance, crates/sketchpad-core/src/layernorm.rs:63-73) vs the oracle.
Metric rel_err = max|gpu - oracle| / max|oracle|: 1e-3 (fp32), 2e-2 (bf16)."""
import numpy as np
import pytest
import torch

import oracle
from sketchpad_b200 import layer_norm
from helpers import TOL_F32, TOL_HALF, rel_err, to_np

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,n", [(8192, 320), (2048, 640), (512, 1280), (77, 768), (5, 3)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_layernorm(rows, n, dtype):
    g = torch.Generator().manual_seed(rows + n)
    x = (torch.randn(rows, n, generator=g) * 2 + 0.3).to(dtype)
    w = (torch.randn(n, generator=g) * 0.1 + 1).to(dtype)
    b = (torch.randn(n, generator=g) * 0.1).to(dtype)
    y = layer_norm(x.cuda(), w.cuda(), b.cuda())
    ref = oracle.layernorm(to_np(x), to_np(w), to_np(b))
    assert rel_err(to_np(y), ref) < (TOL_F32 if dtype == torch.float32 else TOL_HALF)


@pytest.mark.parametrize("rows,n", [(8192, 320), (77, 768), (5, 3)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_layernorm_add(rows, n, dtype):
    # LayerNorm of x + a[column]: the sum rounded to the dtype first, as a separate add would
    g = torch.Generator().manual_seed(rows * 3 + n)
    x = (torch.randn(rows, n, generator=g) * 2 + 0.3).to(dtype)
    a = (torch.randn(n, generator=g) * 0.5).to(dtype)
    w = (torch.randn(n, generator=g) * 0.1 + 1).to(dtype)
    b = (torch.randn(n, generator=g) * 0.1).to(dtype)
    y = layer_norm(x.cuda(), w.cuda(), b.cuda(), add=a.cuda())
    xs = to_np((x + a[None, :]).to(dtype))
    ref = oracle.layernorm(xs, to_np(w), to_np(b))
    assert rel_err(to_np(y), ref) < (TOL_F32 if dtype == torch.float32 else TOL_HALF)


@pytest.mark.parametrize("b,s,n", [(1, 4608, 3072), (2, 300, 5120), (1, 77, 640), (3, 5, 24),
                                   (2, 9, 6000)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_layernorm_modulate(b, s, n, dtype):
    # LN::new(x) * (1 + scale) + shift with scale / shift sliced out of a modulation output
    # [b, 1, k, n] like the Flux blocks (flux.rs:479-481); (2, 9, 6000) takes the generic path
    from sketchpad_b200 import layer_norm_modulate
    g = torch.Generator().manual_seed(b * s + n)
    x = (torch.randn(b, s, n, generator=g) * 2 + 0.3).to(dtype)
    m = (torch.randn(b, 1, 3, n, generator=g) * 0.3).to(dtype)
    shift, scale = m[:, :, 0], m[:, :, 1]
    md = m.cuda()
    y = layer_norm_modulate(x.cuda(), md[:, :, 1], md[:, :, 0])
    ones = np.ones(n, np.float32)
    ln = oracle.layernorm(to_np(x).reshape(b * s, n), ones, np.zeros(n, np.float32))
    ref = ln.reshape(b, s, n) * (1 + to_np(scale)) + to_np(shift)
    assert rel_err(to_np(y), ref) < (TOL_F32 if dtype == torch.float32 else TOL_HALF)
    # neither vector: plain LayerNorm::new
    y0 = layer_norm_modulate(x.cuda())
    assert rel_err(to_np(y0).reshape(b * s, n), ln) < (TOL_F32 if dtype == torch.float32 else TOL_HALF)


def test_layernorm_modulate_rejects_mismatched_vectors():
    from sketchpad_b200 import layer_norm_modulate
    x = torch.zeros(2, 4, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        layer_norm_modulate(x, torch.zeros(3, 1, 64, device="cuda", dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        layer_norm_modulate(x, torch.zeros(2, 1, 64, device="cuda"))  # f32 vs bf16
