"""SD 1.x-shaped UNet denoise step on the GPU (bf16, sm_100a kernels on the hot path) vs the
CPU oracle's fp32 restatement of UNet::forward (crates/sketchpad-unet/src/unet_sd.rs:235-272),
on identical random-init weights (N(0,0.02), seed 0) and inputs.

Metric: rel_err = max|gpu - oracle| / max|oracle| of the predicted noise; bar 2e-2 (bf16
activations).
"""
import numpy as np
import pytest
import torch

from helpers import TOL_HALF, rel_err, to_np
from oracle.unet import OracleUNet
from sketchpad_b200.unet import UNetB200, make_unet_params

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def params():
    return make_unet_params(seed=0)


@pytest.mark.parametrize("gemm", ["cublas", "sp"])
def test_unet_step_matches_oracle(params, gemm):
    # gemm="sp": the step's dense GEMMs on this library's tcgen05 kernel (Bf16Linear)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 4, 64, 64), dtype=np.float32)
    ctx = rng.standard_normal((2, 77, 768), dtype=np.float32)
    t = np.array([999.0, 999.0], np.float32)
    net = UNetB200(params, gemm=gemm)
    with torch.inference_mode():
        y = net(torch.from_numpy(x).cuda(), torch.from_numpy(t).cuda(), torch.from_numpy(ctx).cuda())
    torch.cuda.synchronize()
    ref = OracleUNet(params)(x, t, ctx)
    err = rel_err(to_np(y), ref)
    print(f"unet rel_err={err:.3e}")
    assert y.shape == (2, 4, 64, 64)
    assert err < TOL_HALF
