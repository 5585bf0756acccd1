"""DiT blocks on the GPU kernels vs the oracle (crates/sketchpad-dit/src/flux.rs:325-607,
wan.rs:351-601), per block at reduced width with the real head_dim 128: Q8_0 dequant-GEMMs
(Flux), FP8 dequant-GEMMs (Wan), flash attention (self, joint K/V, spatial, temporal with
S=3, cross with 40 context tokens), unbiased LayerNorm.  bf16 activations:
rel_err = max|gpu - oracle| / max|oracle| < 2e-2."""
import pytest
import torch

import sketchpad_b200.flux as FX
import sketchpad_b200.wan as WN
from dit_weights import SMALL_FLUX, SMALL_WAN, flux_block_weights, wan_block_weights
from helpers import TOL_HALF, rel_err, to_np
from oracle import dit as OD

pytestmark = pytest.mark.gpu


def _inputs(seed, *shapes):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(*s, generator=g).to(torch.bfloat16) for s in shapes]


def _rope(cfg):
    cos, sin = OD.rope_tables(cfg.head_dim, cfg.max_seq_len)
    return cos, sin, torch.from_numpy(cos).cuda().bfloat16(), torch.from_numpy(sin).cuda().bfloat16()


@pytest.mark.parametrize("n_img,n_txt", [(200, 72), (384, 128)])
def test_flux_double_block_vs_oracle(n_img, n_txt):
    cfg = SMALL_FLUX
    img, txt, cond = _inputs(0, (1, n_img, 256), (1, n_txt, 256), (1, 256))
    cos, sin, ct, st = _rope(cfg)
    blk = FX.FluxDoubleBlockB200(11, cfg, "cuda")
    gi, gt = blk.forward(img.cuda(), txt.cuda(), cond.cuda(), ct, st)
    torch.cuda.synchronize()
    ri, rt = OD.flux_double_block(to_np(img), to_np(txt), to_np(cond),
                                  flux_block_weights(blk, False), 2, 128, cos, sin)
    assert rel_err(to_np(gi), ri) < TOL_HALF
    assert rel_err(to_np(gt), rt) < TOL_HALF


def test_flux_single_block_vs_oracle():
    cfg = SMALL_FLUX
    x, cond = _inputs(1, (1, 272, 256), (1, 256))
    cos, sin, ct, st = _rope(cfg)
    blk = FX.FluxSingleBlockB200(12, cfg, "cuda")
    y = blk.forward(x.cuda(), cond.cuda(), ct, st)
    torch.cuda.synchronize()
    ref = OD.flux_single_block(to_np(x), to_np(cond), flux_block_weights(blk, True), 2, 128,
                               cos, sin)
    assert rel_err(to_np(y), ref) < TOL_HALF


@pytest.mark.parametrize("nt,nh,nw", [(3, 4, 6), (5, 8, 20)])
def test_wan_block_vs_oracle(nt, nh, nw):
    cfg = WN.WanConfig(hidden_size=256, num_heads=2, intermediate=512, max_spatial_len=nh * nw,
                       max_temporal_len=nt) if nh * nw > SMALL_WAN.max_spatial_len else SMALL_WAN
    x, ctx, cond = _inputs(2, (1, nt * nh * nw, 256), (1, 40, 256), (1, 256))
    blk = WN.WanBlockB200(3, cfg, "cuda")
    y = blk.forward(x.cuda(), cond.cuda(), ctx.cuda(), nt, nh, nw)
    torch.cuda.synchronize()
    ref = OD.wan_block(to_np(x), to_np(cond), to_np(ctx), wan_block_weights(blk), nt, nh, nw, 2,
                       128, OD.rope_tables(128, cfg.max_spatial_len),
                       OD.rope_tables(128, cfg.max_temporal_len))
    assert rel_err(to_np(y), ref) < TOL_HALF
