"""Host-side wiring of the Flux and Wan block harnesses (sketchpad_b200/flux.py, wan.py):
stream order, modulation slots, RoPE placement, the cross-stream K/V through the attending
stream's qkv weights, the spatial/temporal regrouping.  The CUDA kernels are swapped for
plain torch ops (CPU, fp32), so this checks only the harness against the oracle's
independent restatement (crates/sketchpad-dit/src/flux.rs:325-607, wan.rs:351-601); the
GPU tests check the kernels."""
import numpy as np
import torch
import torch.nn.functional as F

import sketchpad_b200.flux as FX
import sketchpad_b200.quantization as QZ
import sketchpad_b200.quantized_matmul as QM
import sketchpad_b200.wan as WN
from dit_weights import SMALL_FLUX, SMALL_WAN, flux_block_weights, wan_block_weights
from helpers import rel_err, to_np
from oracle import dit as OD

TOL_WIRING = 1e-4  # fp32 torch stand-ins vs fp32 oracle: summation order only


def _q8_forward(self, x, out=None):
    q = self.q.float()
    s = self.scale.view(torch.float16).float().t().repeat_interleave(32, dim=1)  # [N, K]
    y = x.float() @ (q * s).t()
    return y + self.bias.float() if self.bias is not None else y


def _e4m3(w):
    return w.clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)


def _fp8_quantize(t, cfg):
    assert cfg.scale is not None
    data = _e4m3(t.float() / cfg.scale)
    return QZ.Fp8Tensor(data, torch.full((1,), float(cfg.scale)), QZ.Fp8Format.E4M3, tuple(t.shape))


def _fp8_forward(self, x, out=None):
    w = self.weight.data.view(torch.float8_e4m3fn).float() * self.weight.scale.view(-1, 1)
    y = x.float() @ w.t()
    return y + self.bias.float() if self.bias is not None else y


def _ln(x, w, b, eps, unbiased, out=None):
    xf = x.float()
    return (xf - xf.mean(-1, keepdim=True)) / torch.sqrt(xf.var(-1, keepdim=True, unbiased=unbiased) + eps) * w + b


def _sdpa(q, k, v, out=None):
    o = F.scaled_dot_product_attention(q.float(), k.float(), v.float())
    return out.copy_(o) if out is not None else o


def _swiglu(h):
    f = h.shape[-1] // 2
    return F.silu(h[..., :f]) * h[..., f:]


def _patch(monkeypatch):
    monkeypatch.setattr(QM.GpuQuantizedLinear, "forward", _q8_forward)
    monkeypatch.setattr(QM.GpuQuantizedLinear, "__call__", _q8_forward)
    monkeypatch.setattr(QZ.Fp8Linear, "forward", _fp8_forward)
    monkeypatch.setattr(QZ.Fp8Linear, "__call__", _fp8_forward)
    monkeypatch.setattr(QZ, "quantize_fp8", _fp8_quantize)
    monkeypatch.setattr(FX, "layer_norm", _ln)
    monkeypatch.setattr(WN, "layer_norm", _ln)
    monkeypatch.setattr(FX, "flash_attention", _sdpa)
    monkeypatch.setattr(WN, "flash_attention", _sdpa)
    monkeypatch.setattr(FX, "swiglu", _swiglu)
    monkeypatch.setattr(WN, "swiglu", _swiglu)


def test_flux_blocks_wiring_match_oracle(monkeypatch):
    _patch(monkeypatch)
    cfg = SMALL_FLUX
    g = torch.Generator().manual_seed(0)
    img = torch.randn(1, 200, 256, generator=g)
    txt = torch.randn(1, 72, 256, generator=g)
    cond = torch.randn(1, 256, generator=g)
    cos, sin = OD.rope_tables(cfg.head_dim, cfg.max_seq_len)
    ct, st = torch.from_numpy(cos), torch.from_numpy(sin)

    dbl = FX.FluxDoubleBlockB200(11, cfg, "cpu")
    gi, gt = dbl.forward(img, txt, cond, ct, st)
    ri, rt = OD.flux_double_block(img.numpy(), txt.numpy(), cond.numpy(),
                                  flux_block_weights(dbl, False), 2, 128, cos, sin)
    assert rel_err(to_np(gi), ri) < TOL_WIRING
    assert rel_err(to_np(gt), rt) < TOL_WIRING

    sgl = FX.FluxSingleBlockB200(12, cfg, "cpu")
    x = torch.cat([img, txt], dim=1)
    gx = sgl.forward(x, cond, ct, st)
    rx = OD.flux_single_block(x.numpy(), cond.numpy(), flux_block_weights(sgl, True), 2, 128,
                              cos, sin)
    assert rel_err(to_np(gx), rx) < TOL_WIRING


def test_wan_block_wiring_matches_oracle(monkeypatch):
    _patch(monkeypatch)
    cfg = SMALL_WAN
    nt, nh, nw = 3, 4, 6
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1, nt * nh * nw, 256, generator=g)
    ctx = torch.randn(1, 40, 256, generator=g)
    cond = torch.randn(1, 256, generator=g)
    blk = WN.WanBlockB200(3, cfg, "cpu", rope_dtype=torch.float32)
    y = blk.forward(x, cond, ctx, nt, nh, nw)
    ref = OD.wan_block(x.numpy(), cond.numpy(), ctx.numpy(), wan_block_weights(blk), nt, nh, nw,
                       2, 128, OD.rope_tables(128, 64), OD.rope_tables(128, 8))
    assert rel_err(to_np(y), ref) < TOL_WIRING


def test_oracle_rope_matches_reference_rotation():
    # rope.rs:145-170 on a hand case: position 1, head_dim 4 -> pairs rotate by 1 and 1e-2 rad
    cos, sin = OD.rope_tables(4, 2)
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32).reshape(1, 1, 1, 4)
    x2 = np.concatenate([np.zeros_like(x), x], axis=2)  # positions 0 and 1
    y = OD.rope_apply(x2, cos, sin)[0, 0, 1]
    a0, a1 = 1.0, 1.0 / 100.0
    want = [1 * np.cos(a0) - 2 * np.sin(a0), 1 * np.sin(a0) + 2 * np.cos(a0),
            3 * np.cos(a1) - 4 * np.sin(a1), 3 * np.sin(a1) + 4 * np.cos(a1)]
    assert np.allclose(y, want, atol=1e-6)
