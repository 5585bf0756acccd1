"""Convolution bias + residual add (ResBlock::forward, crates/sketchpad-unet/src/blocks.rs:
123-150) in one pass vs the f32 sum of the same rounded inputs.  rel_err = max|gpu - ref| /
max|ref|: 1e-6 for f32 (one rounding), 2e-2 for bf16/f16."""
import numpy as np
import pytest
import torch

from helpers import TOL_HALF, rel_err, to_np
from sketchpad_b200.residual import add_bias_residual

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 320, 64, 64), (2, 1280, 8, 8), (1, 16, 3, 5)])
@pytest.mark.parametrize("with_residual", [True, False])
def test_add_bias_residual(shape, dtype, with_residual):
    g = torch.Generator().manual_seed(3)
    y = torch.randn(*shape, generator=g).to(dtype)
    r = torch.randn(*shape, generator=g).to(dtype)
    b = torch.randn(shape[1], generator=g).to(dtype)
    ref = to_np(y) + to_np(b)[None, :, None, None] + (to_np(r) if with_residual else 0.0)
    cl = torch.channels_last
    out = add_bias_residual(y.cuda().to(memory_format=cl), b.cuda(),
                            r.cuda().to(memory_format=cl) if with_residual else None)
    assert out.is_contiguous(memory_format=cl)
    assert rel_err(to_np(out), ref) < (1e-6 if dtype == torch.float32 else TOL_HALF)


def test_add_bias_residual_rejects_nchw_and_misfit():
    y = torch.zeros(1, 16, 4, 4, device="cuda")
    with pytest.raises(ValueError, match="channels-last"):
        add_bias_residual(y, torch.zeros(16, device="cuda"))
    y = torch.zeros(1, 12, 4, 4, device="cuda", dtype=torch.bfloat16).to(memory_format=torch.channels_last)
    with pytest.raises(Exception, match="multiple"):
        add_bias_residual(y, torch.zeros(12, device="cuda", dtype=torch.bfloat16))
