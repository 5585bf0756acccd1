"""GroupNorm(+SiLU) CUDA kernel vs the CPU oracle (crates/sketchpad-core/src/groupnorm.rs:62-102).

Metric: rel_err = max|gpu - oracle| / max|oracle|; bars: 1e-3 (fp32), 2e-2 (fp16/bf16).
Inputs follow BASELINE config 2: x ~ N(0,1)*3+0.5, gamma ~ N(1,0.1), beta ~ N(0,0.1), seed 0.
For f16/bf16 tensors the oracle runs the reference's dtype path (groupnorm.rs:88-99): the
normalised value cast back to the tensor dtype, then the affine, clamp and SiLU as f16/bf16
tensor ops, each rounded.  The kernel keeps f32 through the affine and SiLU and rounds once.
"""
import numpy as np
import pytest
import torch

import oracle
from sketchpad_b200 import GroupNormSiLuLayer, GroupNormSiLuOptions, groupnorm, groupnorm_silu
from helpers import TOL_F32, TOL_HALF, rel_err, to_np

pytestmark = pytest.mark.gpu


def dt(dtype):
    """The oracle's dtype argument for a torch dtype (None = the f32 path)."""
    return {torch.float32: None, torch.float16: "f16", torch.bfloat16: "bf16"}[dtype]

SHAPES = [(2, 320, 64, 64), (2, 640, 32, 32), (2, 1280, 16, 16), (2, 512, 128, 128),
          (8, 320, 64, 64), (8, 640, 32, 32), (8, 1280, 16, 16), (8, 512, 128, 128)]


def make(shape, seed=0):
    rng = np.random.default_rng(seed)
    B, C, H, W = shape
    x = (rng.standard_normal(shape, dtype=np.float32) * 3 + 0.5).astype(np.float32)
    g = (rng.standard_normal(C, dtype=np.float32) * 0.1 + 1).astype(np.float32)
    b = (rng.standard_normal(C, dtype=np.float32) * 0.1).astype(np.float32)
    return x, g, b


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_groupnorm_silu_baseline_sweep(shape, dtype):
    x, g, b = make(shape)
    xt = torch.from_numpy(x).cuda().to(dtype)
    # the oracle sees exactly the values the GPU sees
    ref = oracle.groupnorm_act(to_np(xt), to_np(torch.from_numpy(g).to(dtype)),
                               to_np(torch.from_numpy(b).to(dtype)), 32, 1e-5, silu=True,
                               dtype=dt(dtype))
    y = groupnorm_silu(xt, torch.from_numpy(g).cuda().to(dtype), torch.from_numpy(b).cuda().to(dtype))
    torch.cuda.synchronize()
    tol = TOL_F32 if dtype == torch.float32 else TOL_HALF
    assert rel_err(to_np(y), ref) < tol


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_groupnorm_without_silu(dtype):
    x, g, b = make((2, 320, 64, 64), seed=1)
    xt = torch.from_numpy(x).cuda().to(dtype)
    gg, bb = torch.from_numpy(g).to(dtype), torch.from_numpy(b).to(dtype)
    ref = oracle.groupnorm_act(to_np(xt), to_np(gg), to_np(bb), 32, 1e-5, silu=False,
                               dtype=dt(dtype))
    y = groupnorm(xt, gg.cuda(), bb.cuda())
    tol = TOL_F32 if dtype == torch.float32 else TOL_HALF
    assert rel_err(to_np(y), ref) < tol


@pytest.mark.parametrize("shape,groups", [((1, 32, 8, 8), 8), ((3, 64, 7, 9), 32),
                                          ((1, 4, 1, 1), 2), ((2, 96, 5, 5), 32),
                                          ((1, 64, 300, 300), 32), ((1, 32, 96, 96), 1)])
def test_groupnorm_ragged_and_general_paths(shape, groups):
    # odd spatial sizes (no 16-byte vectors), tiny groups, and groups too large for one
    # cluster (the two-pass workspace path)
    x, _, _ = make(shape, seed=2)
    C = shape[1]
    rng = np.random.default_rng(3)
    g = rng.uniform(0.5, 1.5, C).astype(np.float32)
    b = rng.uniform(-0.5, 0.5, C).astype(np.float32)
    ref = oracle.groupnorm_act(x, g, b, groups, 1e-5, silu=True)
    y = groupnorm_silu(torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda(),
                       torch.from_numpy(b).cuda(), GroupNormSiLuOptions(groups, 1e-5))
    assert rel_err(to_np(y), ref) < TOL_F32


@pytest.mark.parametrize("shape,groups", [((2, 512, 128, 128), 32), ((1, 48, 100, 100), 3)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_groupnorm_silu_streaming_path_16bit(shape, groups, dtype):
    # 512 KB and 320 KB 16-bit groups take the streaming path: slices inside one channel
    # (128 x 128) and slices straddling channels (100 x 100); SiLU on packed 16-bit pairs
    x, g, b = make(shape, seed=6)
    xt = torch.from_numpy(x).cuda().to(dtype)
    gg, bb = torch.from_numpy(g).to(dtype), torch.from_numpy(b).to(dtype)
    ref = oracle.groupnorm_act(to_np(xt), to_np(gg), to_np(bb), groups, 1e-5, silu=True,
                               dtype=dt(dtype))
    y = groupnorm_silu(xt, gg.cuda(), bb.cuda(), GroupNormSiLuOptions(groups, 1e-5))
    assert rel_err(to_np(y), ref) < TOL_HALF


@pytest.mark.parametrize("shape,groups,offset", [((1, 48, 100, 100), 3, 1000.0),
                                                 ((3, 64, 64, 64), 2, -300.0)])
def test_groupnorm_streaming_path_offset_mean(shape, groups, offset):
    # groups of 640 KB / 2 MB f32 take the persistent streaming path (per-thread sums shifted
    # by the thread's first value, merged across the cluster); a mean far from zero checks
    # that the variance does not cancel
    x, _, _ = make(shape, seed=4)
    x = (x / 3.0 + offset).astype(np.float32)
    C = shape[1]
    rng = np.random.default_rng(5)
    g = rng.uniform(0.5, 1.5, C).astype(np.float32)
    b = rng.uniform(-0.5, 0.5, C).astype(np.float32)
    ref = oracle.groupnorm_act(x, g, b, groups, 1e-5, silu=True)
    y = groupnorm_silu(torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda(),
                       torch.from_numpy(b).cuda(), GroupNormSiLuOptions(groups, 1e-5))
    assert rel_err(to_np(y), ref) < TOL_F32


def test_groupnorm_strided_input():
    # an H/W-transposed view is neither NCHW- nor NHWC-contiguous: the general strided path
    x, g, b = make((2, 64, 16, 24), seed=4)
    xt = torch.from_numpy(x).cuda().transpose(2, 3)
    assert not xt.is_contiguous() and not xt.is_contiguous(memory_format=torch.channels_last)
    ref = oracle.groupnorm_act(np.ascontiguousarray(x.transpose(0, 1, 3, 2)), g, b, 32, 1e-5, silu=True)
    y = groupnorm_silu(xt, torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda())
    assert y.is_contiguous()
    assert rel_err(to_np(y), ref) < TOL_F32


@pytest.mark.parametrize("shape", [(2, 320, 64, 64), (2, 640, 32, 32), (2, 1280, 8, 8),
                                   (2, 2560, 8, 8), (2, 1920, 16, 16), (2, 960, 32, 32),
                                   (1, 64, 300, 300), (3, 96, 7, 9)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_groupnorm_channels_last(shape, dtype):
    # the UNet keeps activations channels-last; output keeps the input's layout
    x, g, b = make(shape, seed=7)
    xt = torch.from_numpy(x).cuda().to(dtype).to(memory_format=torch.channels_last)
    ref = oracle.groupnorm_act(to_np(xt), to_np(torch.from_numpy(g).to(dtype)),
                               to_np(torch.from_numpy(b).to(dtype)), 32, 1e-5, silu=True,
                               dtype=dt(dtype))
    y = groupnorm_silu(xt, torch.from_numpy(g).cuda().to(dtype), torch.from_numpy(b).cuda().to(dtype))
    assert y.is_contiguous(memory_format=torch.channels_last)
    tol = TOL_F32 if dtype == torch.float32 else TOL_HALF
    assert rel_err(to_np(y), ref) < tol
    y2 = groupnorm_silu(xt, torch.from_numpy(g).cuda().to(dtype), torch.from_numpy(b).cuda().to(dtype))
    assert torch.equal(y, y2)  # the ticket counters reset: a second call is identical


@pytest.mark.parametrize("shape", [(2, 320, 64, 64), (2, 1280, 16, 16), (2, 2560, 8, 8)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_groupnorm_add_channels_last(shape, dtype):
    # ResBlock's norm2(h + temb[:, :, None, None]) in one pass: the oracle normalises the
    # explicit sum, rounded to the tensor dtype as the reference's separate add is (the
    # kernel keeps the sum in f32)
    x, g, b = make(shape, seed=11)
    B, C = shape[:2]
    t = np.random.default_rng(12).standard_normal((B, C)).astype(np.float32)
    xt = torch.from_numpy(x).cuda().to(dtype).to(memory_format=torch.channels_last)
    tt = torch.from_numpy(t).cuda().to(dtype)
    xs = to_np(torch.from_numpy(to_np(xt) + to_np(tt)[:, :, None, None]).to(dtype))
    ref = oracle.groupnorm_act(xs, to_np(torch.from_numpy(g).to(dtype)),
                               to_np(torch.from_numpy(b).to(dtype)), 32, 1e-5, silu=True,
                               dtype=dt(dtype))
    y = groupnorm_silu(xt, torch.from_numpy(g).cuda().to(dtype), torch.from_numpy(b).cuda().to(dtype),
                       add=tt)
    assert y.is_contiguous(memory_format=torch.channels_last)
    tol = TOL_F32 if dtype == torch.float32 else TOL_HALF
    assert rel_err(to_np(y), ref) < tol


@pytest.mark.parametrize("shape,groups,dtype", [
    ((1, 4096, 6, 6), 1, torch.bfloat16),   # cooperative single-launch kernel
    ((1, 2048, 6, 6), 1, torch.float32),    # cooperative single-launch kernel
    ((2, 8192, 4, 4), 2, torch.bfloat16),   # stats + apply kernel pair
    ((1, 4096, 6, 6), 1, torch.float32)])   # stats + apply kernel pair
def test_groupnorm_channels_last_fallback_paths(shape, groups, dtype):
    # groups wider than one cluster's channel slice take the fallback channels-last paths
    x, g, b = make(shape, seed=13)
    xt = torch.from_numpy(x).cuda().to(dtype).to(memory_format=torch.channels_last)
    gt, bt = torch.from_numpy(g).to(dtype), torch.from_numpy(b).to(dtype)
    ref = oracle.groupnorm_act(to_np(xt), to_np(gt), to_np(bt), groups, 1e-5, silu=True,
                               dtype=dt(dtype))
    t = torch.from_numpy(np.random.default_rng(14).standard_normal(shape[:2]).astype(np.float32))
    y = groupnorm_silu(xt, gt.cuda(), bt.cuda(), GroupNormSiLuOptions(groups, 1e-5))
    tol = TOL_F32 if dtype == torch.float32 else TOL_HALF
    assert rel_err(to_np(y), ref) < tol
    # and the folded time-embedding add on the same paths
    tt = t.to(dtype)
    xs = to_np(torch.from_numpy(to_np(xt) + to_np(tt)[:, :, None, None]).to(dtype))
    ref2 = oracle.groupnorm_act(xs, to_np(gt), to_np(bt), groups, 1e-5, silu=True,
                                dtype=dt(dtype))
    y2 = groupnorm_silu(xt, gt.cuda(), bt.cuda(), GroupNormSiLuOptions(groups, 1e-5), add=tt.cuda())
    assert rel_err(to_np(y2), ref2) < tol


def test_groupnorm_add_rejects_nchw():
    x = torch.zeros(1, 32, 4, 4, device="cuda")
    with pytest.raises(Exception, match="channels-last"):
        groupnorm_silu(x, torch.ones(32, device="cuda"), torch.zeros(32, device="cuda"),
                       add=torch.zeros(1, 32, device="cuda"))


def test_groupnorm_clamps_large_values():
    x, g, b = make((1, 32, 4, 4), seed=5)
    x[0, 0, 0, 0] = 1e6
    x[0, 5, 1, 1] = -3e5
    ref = oracle.groupnorm_act(x, g, b, 8, 1e-5, silu=False)
    y = groupnorm(torch.from_numpy(x).cuda(), torch.from_numpy(g).cuda(),
                  torch.from_numpy(b).cuda(), GroupNormSiLuOptions(8))
    assert rel_err(to_np(y), ref) < TOL_F32


def test_groupnorm_rejects_indivisible_channels():
    x = torch.zeros(1, 30, 2, 2, device="cuda")
    with pytest.raises(ValueError):
        groupnorm_silu(x, torch.ones(30, device="cuda"), torch.zeros(30, device="cuda"))


def test_groupnorm_layer_api():
    x, g, b = make((2, 640, 32, 32), seed=6)
    layer = GroupNormSiLuLayer.from_tensors(32, torch.from_numpy(g).cuda(), torch.from_numpy(b).cuda())
    ref = oracle.groupnorm_act(x, g, b, 32, 1e-5, silu=True)
    assert rel_err(to_np(layer.forward(torch.from_numpy(x).cuda())), ref) < TOL_F32
