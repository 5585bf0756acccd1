"""GLU gates (GEGLU of the UNet feed-forward, SwiGLU of the Flux/Wan feed-forwards) vs the
oracle's element-wise activations (crates/sketchpad-unet/src/blocks.rs:446-458,
crates/sketchpad-core/src/glu.rs:91-96).  rel_err = max|gpu - oracle| / max|oracle|:
1e-3 for f32, 2e-2 for bf16/f16."""
import numpy as np
import pytest
import torch

import oracle
from helpers import TOL_F32, TOL_HALF, rel_err, to_np
from sketchpad_b200.glu import geglu, swiglu

pytestmark = pytest.mark.gpu


def _hidden(M, F, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(M, 2 * F, generator=g) * 2).to(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,F", [(8192, 1280), (77, 40), (3, 2560)])
def test_geglu_vs_oracle(M, F, dtype):
    h = _hidden(M, F, dtype)
    hn = to_np(h)
    ref = hn[:, :F] * oracle.activation(hn[:, F:], "gelu")
    y = geglu(h.cuda())
    torch.cuda.synchronize()
    assert rel_err(to_np(y), ref) < (TOL_F32 if dtype == torch.float32 else TOL_HALF)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,F", [(4608, 12288), (40, 64)])
def test_swiglu_vs_oracle(M, F, dtype):
    h = _hidden(M, F, dtype, seed=1)
    hn = to_np(h)
    ref = oracle.activation(hn[:, :F], "silu") * hn[:, F:]
    y = swiglu(h.cuda())
    torch.cuda.synchronize()
    assert rel_err(to_np(y), ref) < (TOL_F32 if dtype == torch.float32 else TOL_HALF)


def test_glu_gate_strided_rows_and_errors():
    # a row slice of a wider buffer: x row stride 2F + 16
    F = 64
    base = _hidden(10, F + 8, torch.bfloat16, seed=2).cuda()
    h = base[:, : 2 * F]
    y = geglu(h)
    hn = to_np(h)
    ref = hn[:, :F] * oracle.activation(hn[:, F:], "gelu")
    assert rel_err(to_np(y), ref) < TOL_HALF
    with pytest.raises(Exception, match="multiples"):
        geglu(torch.zeros(4, 2 * 12, device="cuda", dtype=torch.bfloat16))  # F=12 not /8
