"""Host-side wiring of the UNet step harness (sketchpad_b200/unet.py): block order, skip
connections, channels-last layouts and the GEMM form of the 1x1 projections.  The CUDA
kernels are swapped for plain torch ops here (CPU, fp32), so this checks only the harness
against the oracle's independent restatement of UNet::forward
(crates/sketchpad-unet/src/unet_sd.rs:235-272); the GPU test checks the kernels."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import sketchpad_b200.unet as U
from oracle.unet import OracleUNet


def _gn(x, w, b, silu, add=None):
    if add is not None:
        x = x + add[:, :, None, None]
    y = F.group_norm(x.float(), 32, w.float(), b.float(), 1e-5)
    y = F.silu(y) if silu else y
    if x.is_contiguous(memory_format=torch.channels_last) and not x.is_contiguous():
        y = y.contiguous(memory_format=torch.channels_last)
    return y


def _ln(x, w, b, eps, unbiased, out=None, add=None):
    xf = x.float() if add is None else x.float() + add.float()
    return (xf - xf.mean(-1, keepdim=True)) / torch.sqrt(xf.var(-1, keepdim=True, unbiased=unbiased) + eps) * w + b


def _bf16lin_forward(self, x, out=None, gate=None, residual=None, glu=None):
    # Bf16Linear's epilogues in f32 torch: x W^T + b, then the row-interleaved GLU or
    # residual + gate * (...), written into `out` when given
    y = x.reshape(-1, self.in_features).float() @ self.weight.float().t()
    if self.bias is not None:
        y = y + self.bias.float()
    if glu is not None:
        y = y[:, 0::2] * F.gelu(y[:, 1::2])
    else:
        if gate is not None:
            y = y * gate.float().reshape(-1)
        if residual is not None:
            y = y + residual.float().reshape(y.shape)
    y = y.reshape(*x.shape[:-1], y.shape[-1])
    return out.copy_(y.reshape(out.shape)) if out is not None else y


@pytest.mark.parametrize("sp_gemm", [False, True])
def test_unet_harness_wiring_matches_oracle(monkeypatch, sp_gemm):
    # sp_gemm: the dense GEMMs through Bf16Linear and its epilogues (bias, in-place residual,
    # GEGLU over row-interleaved weights, proj_out's folded bias + residual), as on the GPU
    import sketchpad_b200.linear as LIN
    monkeypatch.setattr(LIN.Bf16Linear, "forward", _bf16lin_forward)
    monkeypatch.setattr(U, "groupnorm_silu",
                        lambda x, w, b, opt, out=None, add=None: _gn(x, w, b, True, add))
    monkeypatch.setattr(U, "groupnorm", lambda x, w, b, opt, out=None: _gn(x, w, b, False))
    monkeypatch.setattr(U, "layer_norm", _ln)
    monkeypatch.setattr(U, "geglu", lambda h: h[..., : h.shape[-1] // 2] * F.gelu(h[..., h.shape[-1] // 2:]))
    monkeypatch.setattr(U, "add_bias_residual",
                        lambda y, b, r=None: y + b[None, :, None, None] + (0 if r is None else r))
    monkeypatch.setattr(U, "flash_attention", lambda q, k, v, out=None: out.copy_(
        F.scaled_dot_product_attention(q.float(), k.float(), v.float())))
    P = U.make_unet_params(seed=0)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 4, 64, 64), dtype=np.float32)
    ctx = rng.standard_normal((2, 77, 768), dtype=np.float32)
    t = np.array([999.0, 999.0], np.float32)
    net = U.UNetB200(P, device="cpu", dtype=torch.float32)
    net.sp_gemm = sp_gemm  # the "sp" GEMM path's wiring, on the CPU stand-in above
    with torch.inference_mode():
        y = net(torch.from_numpy(x), torch.from_numpy(t), torch.from_numpy(ctx)).numpy()
    ref = OracleUNet(P)(x, t, ctx)
    assert np.abs(y - ref).max() / np.abs(ref).max() < 1e-4


def test_unet_flops_breakdown():
    f = U.unet_flops()
    assert abs(f["total"] - 1.1285e12) / 1.1285e12 < 1e-3
    assert f["attention"] > 2.3e11
