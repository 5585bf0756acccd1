"""Host-side wiring of the Flux and Wan block harnesses (sketchpad_b200/flux.py, wan.py):
stream order, modulation slots, RoPE placement, the cross-stream K/V through the attending
stream's qkv weights, the spatial/temporal regrouping.  The CUDA kernels are swapped for
plain torch ops (CPU, fp32), so this checks only the harness against the oracle's
independent restatement (crates/sketchpad-dit/src/flux.rs:325-607, wan.rs:351-601); the
GPU tests check the kernels."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import sketchpad_b200.flux as FX
import sketchpad_b200.quantization as QZ
import sketchpad_b200.quantized_matmul as QM
import sketchpad_b200.wan as WN
from dit_weights import (SMALL_FLUX, SMALL_WAN, flux_block_weights, flux_model_weights,
                         wan_block_weights, wan_model_weights)
from helpers import rel_err, to_np
from oracle import dit as OD

TOL_WIRING = 1e-4  # fp32 torch stand-ins vs fp32 oracle: summation order only


def _rope_epilogue(y, rope):
    # RopeEpilogue on rows of y [M, N]: pairs (x0, x1) -> (x0 c - x1 s, x1 c + x0 s)
    M = y.shape[0]
    tab = rope.table.float()
    mod = rope.pos_mod if rope.pos_mod is not None else tab.shape[0]
    pos = ((torch.arange(M) + rope.pos_offset) // rope.pos_div) % mod
    cs = tab[pos]  # [M, D/2, 2]
    heads = y[:, : rope.cols].reshape(M, -1, rope.head_dim // 2, 2)
    x0, x1 = heads[..., 0], heads[..., 1]
    c, s = cs[:, None, :, 0], cs[:, None, :, 1]
    rot = torch.stack((x0 * c - x1 * s, x1 * c + x0 * s), dim=-1).reshape(M, rope.cols)
    return torch.cat([rot, y[:, rope.cols:]], dim=1)


def _epilogue(y, out, gate, residual, rope=None):
    # the GEMM epilogue's residual + gate * rope(y), written into `out` when given
    if rope is not None:
        y = _rope_epilogue(y.reshape(-1, y.shape[-1]), rope).reshape(y.shape)
    if gate is not None:
        y = y * gate.float().reshape(-1)
    if residual is not None:
        y = y + residual.float().reshape(y.shape)
    if out is None:
        return y
    return out.copy_(y.reshape(out.shape))


def _glu(y, glu):
    # the GLU epilogue on row-interleaved columns (lo = even, hi = odd)
    lo, hi = y[..., 0::2], y[..., 1::2]
    return F.silu(lo) * hi if glu == 1 else lo * F.gelu(hi)


def _q8_forward(self, x, out=None, gate=None, residual=None, rope=None, glu=None,
                out_dtype=None):
    q = self.q.float()
    s = self.scale.view(torch.float16).float().t().repeat_interleave(32, dim=1)  # [N, K]
    y = x.float() @ (q * s).t()
    y = y + self.bias.float() if self.bias is not None else y
    if glu is not None:
        return _glu(y, glu)
    return _epilogue(y, out, gate, residual, rope)


def _e4m3(w):
    return w.clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)


def _fp8_quantize(t, cfg):
    assert cfg.scale is not None
    data = _e4m3(t.float() / cfg.scale)
    return QZ.Fp8Tensor(data, torch.full((1,), float(cfg.scale)), QZ.Fp8Format.E4M3, tuple(t.shape))


def _fp8_forward(self, x, out=None, gate=None, residual=None, rope=None, glu=None,
                 out_dtype=None):
    # out_dtype (f16 attention inputs on the GPU) is ignored: the wiring runs in f32
    w = self.weight.data.view(torch.float8_e4m3fn).float() * self.weight.scale.view(-1, 1)
    y = x.float() @ w.t()
    y = y + self.bias.float() if self.bias is not None else y
    if glu is not None:
        return _glu(y, glu)
    return _epilogue(y, out, gate, residual, rope)


def _ln(x, w, b, eps, unbiased, out=None):
    xf = x.float()
    return (xf - xf.mean(-1, keepdim=True)) / torch.sqrt(xf.var(-1, keepdim=True, unbiased=unbiased) + eps) * w + b


def _ln_mod(x, scale=None, shift=None, eps=1e-5, unbiased=True, out=None):
    n = x.shape[-1]
    y = _ln(x, torch.ones(n), torch.zeros(n), eps, unbiased)
    if scale is not None:
        y = y * (1 + scale.float())
    if shift is not None:
        y = y + shift.float()
    return y


def _sdpa(q, k, v, out=None):
    o = F.scaled_dot_product_attention(q.float(), k.float(), v.float())
    return out.copy_(o) if out is not None else o


def _patch(monkeypatch):
    monkeypatch.setattr(QM.GpuQuantizedLinear, "forward", _q8_forward)
    monkeypatch.setattr(QM.GpuQuantizedLinear, "__call__", _q8_forward)
    monkeypatch.setattr(QZ.Fp8Linear, "forward", _fp8_forward)
    monkeypatch.setattr(QZ.Fp8Linear, "__call__", _fp8_forward)
    monkeypatch.setattr(QZ, "quantize_fp8", _fp8_quantize)
    monkeypatch.setattr(FX, "layer_norm_modulate", _ln_mod)
    monkeypatch.setattr(WN, "layer_norm_modulate", _ln_mod)
    monkeypatch.setattr(FX, "flash_attention", _sdpa)
    monkeypatch.setattr(WN, "flash_attention", _sdpa)


@pytest.mark.parametrize("epilogue", [False, True])
def test_flux_blocks_wiring_match_oracle(monkeypatch, epilogue):
    _patch(monkeypatch)
    # epilogue=True routes the gated residual adds through the GEMM-epilogue arguments
    # (the bf16 batch-1 path on the GPU), False through torch element-wise ops
    monkeypatch.setattr(FX, "_epilogue_fusable", lambda r: epilogue)
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


@pytest.mark.parametrize("epilogue", [False, True])
def test_wan_block_wiring_matches_oracle(monkeypatch, epilogue):
    _patch(monkeypatch)
    # epilogue=True applies RoPE through the qkv GEMMs' epilogue arguments (the bf16 path on
    # the GPU), False through apply_rope
    monkeypatch.setattr(WN, "_rope_fusable", lambda x: epilogue)
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


class _Setter:
    # monkeypatch stand-in for spawned ranks (the process ends with the test)
    @staticmethod
    def setattr(obj, name, value):
        setattr(obj, name, value)


def _wan_ulysses_worker(rank, ws, port, result_dir):
    import os
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        _patch(_Setter())
        WN._rope_fusable = lambda x: True  # RoPE by global token index in the qkv epilogue
        cfg = SMALL_WAN
        nt, nh, nw = 3, 4, 6
        g = torch.Generator().manual_seed(1)
        x = torch.randn(1, nt * nh * nw, 256, generator=g)
        ctx = torch.randn(1, 40, 256, generator=g)
        cond = torch.randn(1, 256, generator=g)
        blk = WN.WanBlockB200(3, cfg, "cpu", group=dist.group.WORLD, rope_dtype=torch.float32)
        s = x.shape[1] // ws
        sl = slice(rank * s, (rank + 1) * s)
        y = blk.forward(x[:, sl].contiguous(), cond, ctx, nt, nh, nw)
        ref = OD.wan_block(x.numpy(), cond.numpy(), ctx.numpy(), wan_block_weights(blk), nt, nh,
                           nw, 2, 128, OD.rope_tables(128, 64), OD.rope_tables(128, 8))
        np.save(f"{result_dir}/err{rank}.npy", np.array([rel_err(to_np(y), ref[:, sl])]))
    finally:
        dist.destroy_process_group()


def test_wan_block_ulysses_two_ranks_matches_oracle(tmp_path):
    # sequence-parallel WanBlock (each rank 36 of 72 tokens, one head each): the epilogue RoPE
    # positions count from the rank's first global token (36 -> spatial position 12)
    import socket
    import torch.multiprocessing as mp
    sk = socket.socket()
    sk.bind(("127.0.0.1", 0))
    port = sk.getsockname()[1]
    sk.close()
    mp.spawn(_wan_ulysses_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    errs = [float(np.load(tmp_path / f"err{r}.npy")[0]) for r in range(2)]
    assert max(errs) < TOL_WIRING


def test_flux_model_wiring_matches_oracle(monkeypatch):
    # Flux::forward (flux.rs:686-741): patch embed, text projection, scalar timestep
    # embedding, 1 double + 1 single block, final layer and unpatchify -- the element orders
    # of dit.rs:300-345 followed literally on both sides
    _patch(monkeypatch)
    cfg = SMALL_FLUX
    net = FX.FluxB200(cfg, "cpu", seed=3, num_double=1, num_single=1)
    net.act_dtype = torch.float32
    net.cos, net.sin = (torch.from_numpy(t) for t in OD.rope_tables(cfg.head_dim, cfg.max_seq_len))
    g = torch.Generator().manual_seed(4)
    lat = torch.randn(1, 16, 16, 12, generator=g)
    txt = torch.randn(1, 24, cfg.text_dim, generator=g)
    with torch.no_grad():
        y = net.forward(lat, 0.75, txt)
    W, blocks = flux_model_weights(net)
    W = {k: v for k, v in W.items() if not k.startswith("guidance.")}
    cos, sin = OD.rope_tables(cfg.head_dim, cfg.max_seq_len)
    ref = OD.flux_forward(lat.numpy(), 0.75, txt.numpy(), W, blocks, 1, 1, cfg.num_heads,
                          cfg.head_dim, cfg.patch_size, cos, sin)
    assert y.shape == ref.shape
    assert rel_err(to_np(y), ref) < TOL_WIRING


def test_wan_model_wiring_matches_oracle(monkeypatch):
    # Wan::forward (wan.rs:720-757): patchify, text / time embeddings, 2 blocks, final layer,
    # unpatchify
    _patch(monkeypatch)
    monkeypatch.setattr(WN, "_rope_fusable", lambda x: True)
    cfg = SMALL_WAN
    net = WN.WanB200(cfg, "cpu", seed=5, num_blocks=2)
    net.act_dtype = torch.float32
    for blk in net.blocks:
        blk.s_cos, blk.s_sin, blk.t_cos, blk.t_sin = (
            t.float() for t in (blk.s_cos, blk.s_sin, blk.t_cos, blk.t_sin))
    g = torch.Generator().manual_seed(6)
    lat = torch.randn(1, 16, 3, 8, 12, generator=g)
    txt = torch.randn(1, 20, cfg.text_dim, generator=g)
    with torch.no_grad():
        y = net.forward(lat, 0.5, txt)
    W, blocks = wan_model_weights(net)
    ref = OD.wan_forward(lat.numpy(), 0.5, txt.numpy(), W, blocks, 2, cfg.num_heads,
                         cfg.head_dim, cfg.patch_size, OD.rope_tables(128, cfg.max_spatial_len),
                         OD.rope_tables(128, cfg.max_temporal_len))
    assert y.shape == ref.shape == (1, 16, 3, 8, 12)
    assert rel_err(to_np(y), ref) < TOL_WIRING


def test_oracle_patchify_orders():
    # dit.rs:300-345 / wan.rs:661-718: unpatchify inverts the patch embedding's element order
    # (no projection), and the literal swap orders are not the "[B, ph, pw, C, ps, ps]" the
    # reference's comments describe
    x = np.arange(2 * 4 * 6 * 8, dtype=np.float32).reshape(2, 4, 6, 8)
    p = OD.flux_patch_embed(x, 2)
    assert p.shape == (2, 12, 16)
    v = np.arange(1 * 4 * 3 * 6 * 8, dtype=np.float32).reshape(1, 4, 3, 6, 8)
    pv = OD.wan_patchify(v, 2)
    assert np.array_equal(OD.wan_unpatchify(pv, 3, 3, 4, 4, 2), v)
    # wan's patch k of frame t holds pixels (2*i + a, 2*j + b) of every channel
    assert np.array_equal(pv[0, 0, :4], [v[0, 0, 0, 0, 0], v[0, 0, 0, 0, 1], v[0, 0, 0, 1, 0],
                                         v[0, 0, 0, 1, 1]])


def _wan_model_ulysses_worker(rank, ws, port, result_dir):
    import os
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        _patch(_Setter())
        WN._rope_fusable = lambda x: True
        cfg = SMALL_WAN
        net = WN.WanB200(cfg, "cpu", seed=7, num_blocks=1, group=dist.group.WORLD)
        net.act_dtype = torch.float32
        for blk in net.blocks:
            blk.s_cos, blk.s_sin, blk.t_cos, blk.t_sin = (
                t.float() for t in (blk.s_cos, blk.s_sin, blk.t_cos, blk.t_sin))
        g = torch.Generator().manual_seed(8)
        lat = torch.randn(1, 16, 3, 8, 12, generator=g)
        txt = torch.randn(1, 20, cfg.text_dim, generator=g)
        with torch.no_grad():
            y = net.forward(lat, 0.25, txt)
        W, blocks = wan_model_weights(net)
        ref = OD.wan_forward(lat.numpy(), 0.25, txt.numpy(), W, blocks, 1, cfg.num_heads,
                             cfg.head_dim, cfg.patch_size, OD.rope_tables(128, cfg.max_spatial_len),
                             OD.rope_tables(128, cfg.max_temporal_len))
        np.save(f"{result_dir}/merr{rank}.npy", np.array([rel_err(to_np(y), ref)]))
    finally:
        dist.destroy_process_group()


def test_wan_model_ulysses_two_ranks_matches_oracle(tmp_path):
    # the whole Wan::forward sequence-parallel over 2 gloo ranks: each rank embeds its 36 of
    # 72 tokens; the all-gathered velocity matches the single-device oracle on every rank
    import socket
    import torch.multiprocessing as mp
    sk = socket.socket()
    sk.bind(("127.0.0.1", 0))
    port = sk.getsockname()[1]
    sk.close()
    mp.spawn(_wan_model_ulysses_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    errs = [float(np.load(tmp_path / f"merr{r}.npy")[0]) for r in range(2)]
    assert max(errs) < TOL_WIRING
