"""Ulysses sequence parallelism on GPUs (NCCL all-to-all): a Wan block whose tokens are split
over P ranks gives the same result as the block on one GPU.  Each row of every GEMM,
LayerNorm and attention head is computed by the same kernels in the same order either way,
so the shards are expected to match the single-GPU output to rounding-free agreement; the
bar written here is rel_err < 1e-3.  Runs on 2..8 GPUs (skipped with fewer than 2)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

NT, NH, NW = 4, 8, 16  # 512 tokens: 4 frames of 8 x 16


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    import datetime

    import torch.distributed as dist

    from sketchpad_b200.wan import WanBlockB200, WanConfig

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        cfg = WanConfig(hidden_size=1024, num_heads=8, intermediate=1024,
                        max_spatial_len=NH * NW, max_temporal_len=NT)
        S = NT * NH * NW
        g = torch.Generator().manual_seed(0)
        x = torch.randn(1, S, 1024, generator=g).to(torch.bfloat16).cuda()
        ctx = torch.randn(1, 40, 1024, generator=g).to(torch.bfloat16).cuda()
        cond = torch.randn(1, 1024, generator=g).to(torch.bfloat16).cuda()
        s = S // world
        blk = WanBlockB200(7, cfg, "cuda", group=dist.group.WORLD)
        y = blk.forward(x[:, rank * s:(rank + 1) * s].contiguous(), cond, ctx, NT, NH, NW)
        parts = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(parts, y.contiguous())
        if rank == 0:
            ref = WanBlockB200(7, cfg, "cuda").forward(x, cond, ctx, NT, NH, NW)
            full = torch.cat(parts, dim=1)
            err = ((full.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
            exact = bool(torch.equal(full, ref))
            with open(os.path.join(result_dir, "result.txt"), "w") as f:
                f.write(f"{err} {int(exact)}\n")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_ulysses_wan_block_matches_single_gpu(tmp_path):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = 8 if n >= 8 else (4 if n >= 4 else 2)
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    err, exact = open(tmp_path / "result.txt").read().split()
    print(f"ulysses P={world}: rel_err {err}, bit-identical {exact == '1'}")
    assert float(err) < 1e-3
