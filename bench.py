#!/usr/bin/env python
"""Benchmark: SD 1.x-shaped UNet denoise steps/s on B200, plus the hot-path kernel rooflines.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    (N > 1: python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...)

Workload (on the GPU): one denoise step of the reference's random-init
UNet::new(UNetConfig::sd1x()) for one CFG pair -- batch 2, latent 2x4x64x64 ~ N(0,1), text
context 2x77x768 ~ N(0,1), timestep 999, weights ~ N(0, 0.02) -- in bf16 with the package's
sm_100a GroupNorm(+SiLU), flash attention and LayerNorm kernels (convs/linears: cuDNN/cuBLAS).
Each rank runs its own CFG pair (weak scaling, no collective); value = total steps/s.
The UNet's ~1.2 GB of weights are re-read every step, so the working set exceeds L2.

Prints ONE JSON line on rank 0.  --impl reference times the CPU restatement of the
reference's ndarray path (oracle/, C++/OpenMP) on this host's cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "denoise steps/s at 1/2/4/8 B200; attn TFLOP/s & GN-SiLU GB/s vs roofline"


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as fh:
            d = json.load(fh)
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        for line in (self.out or "").splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------------------
# CPU arms
# ------------------------------------------------------------------------------------------
def cpu_unet_step_time(max_seconds: float = 60.0, min_steps: int = 1, max_steps: int = 1):
    """Seconds per full UNet step of the CPU oracle on this host's cores (bounded sample)."""
    import numpy as np
    import torch

    import oracle
    from oracle.unet import OracleUNet
    from sketchpad_b200.unet import make_unet_params

    oracle.set_threads(os.cpu_count() or 1)
    params = {k: v.numpy() for k, v in make_unet_params(device="cpu").items()}
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 4, 64, 64), dtype=np.float32)
    ctx = rng.standard_normal((2, 77, 768), dtype=np.float32)
    t = np.array([999.0, 999.0], np.float32)
    net = OracleUNet(params)
    times = []
    t_start = time.perf_counter()
    while len(times) < max_steps:
        t0 = time.perf_counter()
        net(x, t, ctx)
        times.append(time.perf_counter() - t0)
        if len(times) >= min_steps and time.perf_counter() - t_start > max_seconds:
            break
    del torch
    return sum(times) / len(times), len(times), oracle.get_threads()


# dram__bytes_read.sum + dram__bytes_write.sum of one (2,8,4096,40) attention launch (ncu
# capture of `bench.py --case attn_2x8x4096x40`): Q, K and V read once, O left in L2
ATTN_D40_TRAFFIC_BYTES = 15_822_592


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    # one warm-up step is skipped when W would push the run past a few minutes; every
    # timed step is one full CFG-pair UNet step of the CPU restatement
    steps = max(1, min(args.steps, 3))
    sec, n, cores = cpu_unet_step_time(max_seconds=150.0, min_steps=1, max_steps=steps)
    value = 1.0 / sec
    line = {
        "metric": METRIC, "impl": "reference", "value": value, "unit": "steps/s",
        "n_gpus": ws, "steps": n, "warmup": 0, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "sd1x_unet_step_cfg_pair", "global_batch": 2, "latent": [4, 64, 64],
                   "context": [77, 768], "timestep": 999, "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "steps/s", "cores": cores, "kind": "port",
                         "sample": f"{n} full UNet step(s) of the C++/OpenMP restatement of the "
                                   "reference ndarray path (oracle/), batch 2"},
        "e2e": {"value": value, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------
def kernel_microbench(torch, peaks, reps=20):
    """Isolated launches of the two headline kernels at their BASELINE sizes (inputs > L2)."""
    from sketchpad_b200 import flash_attention, groupnorm_bytes, groupnorm_silu
    out = {}
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    B, H, S, D = 8, 24, 4608, 128
    q = torch.randn(B, H, S, D, device=dev, generator=g, dtype=torch.bfloat16)
    k = torch.randn(B, H, S, D, device=dev, generator=g, dtype=torch.bfloat16)
    v = torch.randn(B, H, S, D, device=dev, generator=g, dtype=torch.bfloat16)
    o = torch.empty_like(q)
    for _ in range(3):
        flash_attention(q, k, v, out=o)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(reps):
        flash_attention(q, k, v, out=o)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / reps
    fl = 4.0 * B * H * S * S * D
    out["attention_8x24x4608x128"] = {"tflops": fl / ms / 1e9, "ms": ms,
                                      "frac": fl / ms / 1e9 / peaks["bf16_tflops"]}
    del q, k, v, o
    for dt, name in ((torch.float32, "f32"), (torch.float16, "f16")):
        x = (torch.randn(8, 512, 128, 128, device=dev, generator=g) * 3 + 0.5).to(dt)
        w = torch.ones(512, device=dev, dtype=dt)
        b = torch.zeros(512, device=dev, dtype=dt)
        y = torch.empty_like(x)
        for _ in range(3):
            groupnorm_silu(x, w, b, out=y)
        torch.cuda.synchronize()
        s.record()
        for _ in range(reps):
            groupnorm_silu(x, w, b, out=y)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / reps
        by = groupnorm_bytes(8, 512, 128, 128, x.element_size())
        out[f"groupnorm_silu_8x512x128x128_{name}"] = {"gbs": by / ms / 1e6, "ms": ms,
                                                        "frac": by / ms / 1e6 / peaks["hbm_gbs"]}
        del x, y
    return out


def ulysses_wan_block_bench(torch, dist, ws, rank, steps=4, warmup=3):
    """The Wan block at full width (hidden 5120, 40 heads, FFN 13824, FP8 weights) over the
    whole 21 x 45 x 80 = 75,600-token sequence, sequence-parallel (Ulysses) over the ws ranks
    through the library's NCCL communicator (sp_ulysses_a2a): block ms (max over ranks), the
    all-to-all ms inside it (CUDA events around each exchange, max over ranks), its share, and
    the per-GPU bytes sent over NVLink per ms."""
    from sketchpad_b200.comm import NcclComm
    from sketchpad_b200.wan import WanBlockB200, WanConfig, wan_block_flops
    cfg = WanConfig()
    nt, nh, nw = 21, 45, 80
    S = nt * nh * nw
    comm = NcclComm.from_group(timeout=120.0)
    try:
        blk = WanBlockB200(0, cfg, "cuda", group=comm)
        g = torch.Generator(device="cuda").manual_seed(7)
        s = S // ws
        x = torch.randn(1, S, cfg.hidden_size, device="cuda", generator=g).to(torch.bfloat16)
        x = x[:, rank * s:(rank + 1) * s].contiguous()
        ctx = torch.randn(1, 512, cfg.hidden_size, device="cuda", generator=g).to(torch.bfloat16)
        cond = torch.randn(1, cfg.hidden_size, device="cuda", generator=g).to(torch.bfloat16)
        with torch.inference_mode():
            for _ in range(warmup):
                blk.forward(x, cond, ctx, nt, nh, nw)
            comm.wait(120.0)
            dist.barrier()
            torch.cuda.synchronize()
            comm.events = []
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(steps):
                blk.forward(x, cond, ctx, nt, nh, nw)
            b.record()
            comm.wait(120.0)
            torch.cuda.synchronize()
            block_ms = a.elapsed_time(b) / steps
            ev, comm.events = comm.events, None
            a2a_ms = sum(e0.elapsed_time(e1) for e0, e1, _ in ev) / steps
            sent = sum(n for _, _, n in ev) / steps
        t = torch.tensor([block_ms, a2a_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        block_ms, a2a_ms = float(t[0]), float(t[1])
        return {"tokens": S, "ranks": ws, "block_ms": block_ms, "a2a_ms": a2a_ms,
                "a2a_share": a2a_ms / block_ms, "a2a_per_block": len(ev) // steps,
                "a2a_bytes_sent_per_gpu": sent, "a2a_gbs_per_gpu": sent / a2a_ms / 1e6,
                "block_tflops_per_gpu": wan_block_flops(cfg)["total"] / ws / block_ms / 1e9,
                "transport": "sp_ulysses_a2a (library NCCL communicator, grouped send/recv)",
                "timing": "CUDA events around the block and each all-to-all; max over ranks"}
    finally:
        comm.destroy()


def cfg_split_bench(torch, dist, ws, rank, net, steps=10, warmup=3):
    """One CFG pair split over ranks 0 and 1 (the unconditional and the conditional
    prediction, batch 1 each): the pair's step latency is the slower half plus the exchange
    of the two noise predictions (an all-gather of 4x64x64 f32).  Every rank runs its batch-1
    half; the latency reported is that of ranks 0 and 1 (max over all ranks)."""
    from sketchpad_b200.unet import UNetStepGraph
    graph = UNetStepGraph(net, batch=1, warmup=2)
    g = torch.Generator(device="cuda").manual_seed(30 + rank)
    graph.x.copy_(torch.randn(1, 4, 64, 64, device="cuda", generator=g))
    graph.t.fill_(999.0)
    graph.ctx.copy_(torch.randn(1, 77, 768, device="cuda", generator=g))
    eps_all = torch.empty(ws, 1, 4, 64, 64, device="cuda")
    with torch.inference_mode():
        for _ in range(warmup):
            dist.all_gather_into_tensor(eps_all, graph.replay().float())
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            dist.all_gather_into_tensor(eps_all, graph.replay().float())
        b.record()
        torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    t = torch.tensor([ms], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del graph
    return {"pair_step_ms": float(t[0]), "pairs_per_s": 1e3 / float(t[0]),
            "split": "uncond on rank 0, cond on rank 1 (batch 1 each), eps all-gathered",
            "timing": "CUDA events, max over ranks"}


def run_b200(args):
    import torch
    import torch.distributed as dist

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300))
    dev = torch.device("cuda", local)
    peaks, peak_src = load_peaks()

    import sketchpad_b200
    from sketchpad_b200.unet import UNetB200, UNetStepGraph, make_unet_params, unet_flops

    sketchpad_b200.load_library()
    net = UNetB200(make_unet_params(device=dev, seed=0), device=dev)
    g = torch.Generator(device=dev).manual_seed(1 + rank)
    x = torch.randn(2, 4, 64, 64, device=dev, generator=g)
    ctx = torch.randn(2, 77, 768, device=dev, generator=g)
    t = torch.full((2,), 999.0, device=dev)
    flops = unet_flops()

    with torch.inference_mode():
        for _ in range(args.warmup):
            net(x, t, ctx)
        torch.cuda.synchronize()

        # The whole step is captured once as a CUDA graph (the eager step issues ~1000
        # launches); replays run the identical kernels on the same resident buffers.
        graph = None
        step = lambda: net(x, t, ctx)  # noqa: E731
        launches_per_step = None
        if not args.no_graph:
            try:
                graph = UNetStepGraph(net, warmup=2)
                graph.x.copy_(x)
                graph.t.copy_(t)
                graph.ctx.copy_(ctx)
                launches_per_step = graph.kernel_launches
                step = graph.replay
                for _ in range(args.warmup):
                    step()
                torch.cuda.synchronize()
            except Exception as exc:  # capture unsupported: time the eager step instead
                print(f"[bench] graph capture failed, timing eager steps: {exc}", file=sys.stderr)
                graph = None
                step = lambda: net(x, t, ctx)  # noqa: E731

        # ---------------- timed region: inputs resident in HBM ----------------
        launches0 = net.kernel_launches
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            s.record()
            for _ in range(args.steps):
                step()
            e.record()
            torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        ms = s.elapsed_time(e) / args.steps
        if launches_per_step is None:
            launches_per_step = (net.kernel_launches - launches0) // args.steps

        # ---------------- attention inside the step: a second capture of the same step with
        # event-record nodes around each of its attention launches (no CPU gaps in the
        # intervals); replayed step by step, each replay read back before the next
        attn_ms = attn_flops = 0.0
        attn_launches = 0
        eager_ms = None
        try:
            gt = UNetStepGraph(net, warmup=1, time_attention=True)
            gt.x.copy_(x)
            gt.t.copy_(t)
            gt.ctx.copy_(ctx)
            for _ in range(2):
                gt.replay()
            torch.cuda.synchronize()
            for _ in range(args.steps):
                gt.replay()
                torch.cuda.synchronize()
                a_ms, a_fl = gt.attention_ms()
                attn_ms += a_ms
                attn_flops += a_fl
                attn_launches += len(gt.attn_events)
            attn_timing = "event-record nodes around each attention launch in a captured step"
            del gt
        except Exception as exc:
            print(f"[bench] instrumented capture failed, timing attention eagerly: {exc}",
                  file=sys.stderr)
            net.attn_events = []
            torch.cuda.synchronize()
            s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s3.record()
            for _ in range(args.steps):
                net(x, t, ctx)
            e3.record()
            torch.cuda.synchronize()
            eager_ms = s3.elapsed_time(e3) / args.steps
            attn = net.attn_events
            net.attn_events = None
            attn_ms = sum(a.elapsed_time(b) for a, b, _ in attn)
            attn_flops = sum(f for _, _, f in attn)
            attn_launches = len(attn)
            attn_timing = "CUDA events around each attention launch in eager steps"
        attn_launch_ms = attn_ms / max(1, attn_launches)
        attn_share = attn_ms / (ms * args.steps)

        # ---------------- end to end: host buffers through the public API ----------------
        xh = torch.randn(2, 4, 64, 64, generator=torch.Generator().manual_seed(2)).pin_memory()
        ch = torch.randn(2, 77, 768, generator=torch.Generator().manual_seed(3)).pin_memory()
        th = torch.full((2,), 999.0).pin_memory()
        yh = torch.empty(2, 4, 64, 64, dtype=torch.bfloat16).pin_memory()
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record()
        for _ in range(args.steps):
            if graph is not None:
                y = graph(xh, th, ch)  # host buffers in, captured step, host buffer out
            else:
                y = net(xh.to(dev, non_blocking=True), th.to(dev, non_blocking=True),
                        ch.to(dev, non_blocking=True))
            yh.copy_(y, non_blocking=True)
        e2.record()
        torch.cuda.synchronize()
        e2e_ms = s2.elapsed_time(e2) / args.steps
        h2d = xh.numel() * 4 + ch.numel() * 4 + th.numel() * 4
        d2h = yh.numel() * 2

    # max over ranks
    ulysses = cfg_split = None
    if ws > 1:
        tt = torch.tensor([ms, e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(tt[0]), float(tt[1])
        if not args.no_ulysses:
            del graph
            graph = None
            torch.cuda.empty_cache()
            if ws == 2:
                cfg_split = cfg_split_bench(torch, dist, ws, rank, net)
            ulysses = ulysses_wan_block_bench(torch, dist, ws, rank)

    kernels = None
    cpu = None
    if rank == 0:
        kernels = kernel_microbench(torch, peaks)
        if ws == 1 and not args.no_cpu_baseline:
            sec, n, cores = cpu_unet_step_time(max_seconds=30.0, min_steps=1, max_steps=1)
            cpu = {"value": 1.0 / sec, "unit": "steps/s", "cores": cores, "kind": "port",
                   "sample": f"{n} full CFG-pair UNet step of the C++/OpenMP restatement of the "
                             "reference ndarray path (oracle/), fp32"}

    if rank == 0:
        achieved = attn_flops / max(attn_ms, 1e-9) / 1e9  # TFLOP/s
        line = {
            "metric": METRIC, "value": ws * 1e3 / ms, "unit": "steps/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights N(0,0.02), N(0,1) latents/context)",
            "config": {"workload": "sd1x_unet_step_cfg_pair", "global_batch": 2 * ws,
                       "latent": [4, 64, 64], "context": [77, 768], "timestep": 999,
                       "parallelism": f"dp{ws} (independent CFG pairs)",
                       "l2": "working set > L2 (1.2 GB of weights re-read per step)",
                       "step_tflop": flops["total"] / 1e12},
            "e2e": {"value": ws * 1e3 / e2e_ms, "unit": "steps/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * args.steps,
            "cuda_graph": not args.no_graph,
            "roofline": {"kernel": "sp flash attention (all 32 launches of the step)",
                         "bound": "tensor", "achieved": achieved,
                         "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                         "frac": achieved / peaks["bf16_tflops_sustained"],
                         "peak_source": f"{peak_src} bf16_tflops_sustained",
                         "launch_ms": attn_launch_ms, "share_of_step": attn_share,
                         "timing": attn_timing,
                         # ncu dram read+write of one (2,8,4096,40) self-attention launch
                         # (the step's dominant attention shape): Q+K+V read once, O left
                         # in L2 -- equal to the algorithmic input bytes (15.7 MB)
                         "traffic": ATTN_D40_TRAFFIC_BYTES,
                         "traffic_case": "one (2,8,4096,40) launch, ncu dram read + write"},
            "achieved_step_tflops": flops["total"] / ms / 1e9,
            "kernels": kernels,
            "cpu_baseline": cpu,
        }
        if ulysses is not None:
            line["ulysses_wan_block"] = ulysses
        if cfg_split is not None:
            line["cfg_split_pair"] = cfg_split
        line["clocks"] = clk.summary()
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------------------------------
# Single-kernel cases (the workloads the ncu captures run)
# ------------------------------------------------------------------------------------------
def _case_attention(torch, B, H, Sq, Skv, D):
    from sketchpad_b200 import flash_attention
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, H, Sq, D, device="cuda", generator=g, dtype=torch.bfloat16)
    k = torch.randn(B, H, Skv, D, device="cuda", generator=g, dtype=torch.bfloat16)
    v = torch.randn(B, H, Skv, D, device="cuda", generator=g, dtype=torch.bfloat16)
    o = torch.empty(B, H, Sq, D, device="cuda", dtype=torch.bfloat16)
    return (lambda: flash_attention(q, k, v, out=o)), 4.0 * B * H * Sq * Skv * D, "flop"


def _case_attention_short(torch, HW, H, T, D):
    # Wan's temporal attention: [T, HW, H, D] activations viewed as [HW, H, T, D] (strided)
    from sketchpad_b200 import flash_attention
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(T, HW, H, D, device="cuda", generator=g, dtype=torch.bfloat16)
               .permute(1, 2, 0, 3) for _ in range(3))
    o = torch.empty(T, HW, H, D, device="cuda", dtype=torch.bfloat16).permute(1, 2, 0, 3)
    # HBM bytes: q, k, v read once, o written once
    return (lambda: flash_attention(q, k, v, out=o)), 4.0 * T * HW * H * D * 2, "byte"


def _case_groupnorm(torch, B, C, Hh, W, dt):
    from sketchpad_b200 import groupnorm_bytes, groupnorm_silu
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(B, C, Hh, W, device="cuda", generator=g) * 3 + 0.5).to(dt)
    w = torch.ones(C, device="cuda", dtype=dt)
    b = torch.zeros(C, device="cuda", dtype=dt)
    y = torch.empty_like(x)
    return (lambda: groupnorm_silu(x, w, b, out=y)), groupnorm_bytes(B, C, Hh, W, x.element_size()), "byte"


def _case_groupnorm_nhwc(torch, B, C, Hh, W, dt):
    """Channels-last GroupNorm+SiLU as the UNet step calls it (bf16, NHWC)."""
    from sketchpad_b200 import groupnorm_bytes, groupnorm_silu
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(B, C, Hh, W, device="cuda", generator=g) * 3 + 0.5).to(dt)
    x = x.contiguous(memory_format=torch.channels_last)
    w = torch.ones(C, device="cuda", dtype=dt)
    b = torch.zeros(C, device="cuda", dtype=dt)
    y = torch.empty_like(x)
    return (lambda: groupnorm_silu(x, w, b, out=y)), groupnorm_bytes(B, C, Hh, W, x.element_size()), "byte"


def _case_q8(torch, M, N, K):
    from sketchpad_b200.flux import _q8_linear
    lin = _q8_linear(0, N, K, "cuda", bias=True)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    return (lambda: lin.forward(x, out=y)), 2.0 * M * N * K, "flop"


def _case_kquant(torch, name, M, N, K):
    from sketchpad_b200.quantized_matmul import (GpuQuantType, GpuQuantizedLinear,
                                                 make_kquant_synthetic)
    qt = GpuQuantType[name]
    lin = GpuQuantizedLinear.from_bytes(make_kquant_synthetic(qt, N, K), qt, N, K)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    return (lambda: lin.forward(x, out=y)), 2.0 * M * N * K, "flop"


def _case_bf16(torch, M, N, K, cublas=False):
    """One bf16 linear with bias (a UNet projection / feed-forward shape) on this library's
    tcgen05 GEMM, or on cuBLAS (torch.addmm) for comparison."""
    from sketchpad_b200.linear import Bf16Linear
    w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
    b = (torch.randn(N, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    if cublas:
        wt = w.t().contiguous()
        return (lambda: torch.addmm(b, x, wt, out=y)), 2.0 * M * N * K, "flop"
    lin = Bf16Linear(w, b)
    return (lambda: lin.forward(x, out=y)), 2.0 * M * N * K, "flop"


def _case_fp8(torch, M, N, K):
    from sketchpad_b200.wan import fp8_linear_synthetic
    lin = fp8_linear_synthetic(0, N, K, "cuda", bias=True)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    return (lambda: lin.forward(x, out=y)), 2.0 * M * N * K, "flop"


def _case_denoise_loop(torch, kind, steps):
    from sketchpad_b200.denoise import Sd1xDenoiseLoop
    from sketchpad_b200.samplers import DdimSampler, DpmPlusPlusSampler, NoiseSchedule
    from sketchpad_b200.unet import UNetB200, make_unet_params, unet_flops
    net = UNetB200(make_unet_params(device="cuda", seed=0), device="cuda")
    sch = NoiseSchedule.sd1x()
    smp = DdimSampler(sch, steps) if kind == "ddim" else DpmPlusPlusSampler(sch, steps)
    loop = Sd1xDenoiseLoop(net, smp, guidance=7.5)
    g = torch.Generator(device="cuda").manual_seed(1)
    lat = torch.randn(1, 4, 64, 64, device="cuda", generator=g)
    cu = torch.randn(1, 77, 768, device="cuda", generator=g)
    cc = torch.randn(1, 77, 768, device="cuda", generator=g)
    return (lambda: loop(lat, cu, cc)), steps * unet_flops()["total"], "flop"


def _case_unet_step(torch, gemm="cublas"):
    from sketchpad_b200.unet import UNetB200, make_unet_params, unet_flops
    net = UNetB200(make_unet_params(device="cuda", seed=0), device="cuda", gemm=gemm)
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(2, 4, 64, 64, device="cuda", generator=g)
    ctx = torch.randn(2, 77, 768, device="cuda", generator=g)
    t = torch.full((2,), 999.0, device="cuda")

    def step():
        with torch.inference_mode():
            net(x, t, ctx)
    return step, unet_flops()["total"], "flop"


def _case_unet_step_graph(torch, gemm="cublas"):
    """The bench's captured UNet step (CUDA-graph replay of one CFG-pair step) with the given
    GEMM backend: "cublas" (torch matmuls) or "sp" (this library's tcgen05 kernels)."""
    from sketchpad_b200.unet import UNetB200, UNetStepGraph, make_unet_params, unet_flops
    net = UNetB200(make_unet_params(device="cuda", seed=0), device="cuda", gemm=gemm)
    graph = UNetStepGraph(net, warmup=2)
    g = torch.Generator(device="cuda").manual_seed(1)
    graph.x.copy_(torch.randn(2, 4, 64, 64, device="cuda", generator=g))
    graph.ctx.copy_(torch.randn(2, 77, 768, device="cuda", generator=g))
    graph.t.fill_(999.0)
    return graph.graph.replay, unet_flops()["total"], "flop"


def _case_flux_block(torch, single: bool):
    from sketchpad_b200.flux import (FluxConfig, FluxDoubleBlockB200, FluxSingleBlockB200,
                                     flux_step_flops, rope_tables)
    cfg = FluxConfig()
    g = torch.Generator(device="cuda").manual_seed(1)
    rnd = lambda *s: torch.randn(*s, device="cuda", generator=g).to(torch.bfloat16)  # noqa: E731
    cos, sin = (torch.from_numpy(t).to("cuda", torch.bfloat16) for t in rope_tables(128, 4608))
    cond = rnd(1, cfg.hidden_size)
    if single:
        blk, x = FluxSingleBlockB200(7, cfg, "cuda"), rnd(1, 4608, cfg.hidden_size)
        return (lambda: blk.forward(x, cond, cos, sin)), flux_step_flops(cfg, num_double=0, num_single=1), "flop"
    blk = FluxDoubleBlockB200(7, cfg, "cuda")
    img, txt = rnd(1, 4096, cfg.hidden_size), rnd(1, 512, cfg.hidden_size)
    return (lambda: blk.forward(img, txt, cond, cos, sin)), flux_step_flops(cfg, num_double=1, num_single=0), "flop"


def _case_flux_step(torch):
    from sketchpad_b200.flux import FluxB200, FluxConfig, flux_step_flops
    cfg = FluxConfig()
    net = FluxB200(cfg, "cuda", seed=0)
    g = torch.Generator(device="cuda").manual_seed(1)
    lat = torch.randn(1, 16, 128, 128, device="cuda", generator=g)
    txt = torch.randn(1, 512, cfg.text_dim, device="cuda", generator=g).to(torch.bfloat16)
    return (lambda: net.forward(lat, 1.0, txt)), flux_step_flops(cfg), "flop"


def _case_wan_block(torch):
    from sketchpad_b200.wan import WanBlockB200, WanConfig, wan_block_flops
    cfg = WanConfig()
    blk = WanBlockB200(0, cfg, "cuda")
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(1, 21 * 45 * 80, cfg.hidden_size, device="cuda", generator=g).to(torch.bfloat16)
    ctx = torch.randn(1, 512, cfg.hidden_size, device="cuda", generator=g).to(torch.bfloat16)
    cond = torch.randn(1, cfg.hidden_size, device="cuda", generator=g).to(torch.bfloat16)
    return (lambda: blk.forward(x, cond, ctx, 21, 45, 80)), wan_block_flops(cfg)["total"], "flop"


def _case_wan_step(torch):
    """Wan::forward at config 5 on one GPU: 40 FP8 blocks over 21 x 45 x 80 = 75,600 tokens,
    512 text tokens of width 4096, patchify / embeddings / final layer / unpatchify."""
    from sketchpad_b200.wan import WanB200, WanConfig, wan_step_flops
    cfg = WanConfig()
    net = WanB200(cfg, "cuda", seed=0)
    g = torch.Generator(device="cuda").manual_seed(1)
    lat = torch.randn(1, 16, 21, 90, 160, device="cuda", generator=g)
    txt = torch.randn(1, 512, cfg.text_dim, device="cuda", generator=g).to(torch.bfloat16)

    def step():
        with torch.inference_mode():
            net.forward(lat, 0.5, txt)
    return step, wan_step_flops(cfg), "flop"


CASES = {
    "unet_step_eager": _case_unet_step,
    "unet_step_eager_sp_gemm": lambda t: _case_unet_step(t, "sp"),
    "unet_step_graph_cublas": lambda t: _case_unet_step_graph(t, "cublas"),
    "bf16_8192x320x320": lambda t: _case_bf16(t, 8192, 320, 320),
    "bf16_8192x320x320_cublas": lambda t: _case_bf16(t, 8192, 320, 320, True),
    "bf16_8192x2560x320": lambda t: _case_bf16(t, 8192, 2560, 320),
    "bf16_8192x2560x320_cublas": lambda t: _case_bf16(t, 8192, 2560, 320, True),
    "bf16_8192x320x1280": lambda t: _case_bf16(t, 8192, 320, 1280),
    "bf16_8192x320x1280_cublas": lambda t: _case_bf16(t, 8192, 320, 1280, True),
    "unet_step_graph_sp_gemm": lambda t: _case_unet_step_graph(t, "sp"),
    "sd1x_ddim_loop_20": lambda t: _case_denoise_loop(t, "ddim", 20),
    "sd1x_dpmpp2m_loop_20": lambda t: _case_denoise_loop(t, "dpmpp_2m", 20),
    "flux_double_4096x512": lambda t: _case_flux_block(t, False),
    "flux_single_4608": lambda t: _case_flux_block(t, True),
    "flux_step": _case_flux_step,
    "wan_block_21x45x80": _case_wan_block,
    "wan_step_21x45x80": _case_wan_step,
    "attn_8x24x4608x128": lambda t: _case_attention(t, 8, 24, 4608, 4608, 128),
    "attn_2x8x4096x40": lambda t: _case_attention(t, 2, 8, 4096, 4096, 40),
    "attn_2x10x1024x64": lambda t: _case_attention(t, 2, 10, 1024, 1024, 64),
    "attn_cross_2x8x4096x77x40": lambda t: _case_attention(t, 2, 8, 4096, 77, 40),
    "attn_short_3600x40x21x128": lambda t: _case_attention_short(t, 3600, 40, 21, 128),
    "attn_short_900x40x21x128": lambda t: _case_attention_short(t, 900, 40, 21, 128),
    "gn_8x512x128x128_f32": lambda t: _case_groupnorm(t, 8, 512, 128, 128, t.float32),
    "gn_8x512x128x128_f16": lambda t: _case_groupnorm(t, 8, 512, 128, 128, t.float16),
    "gn_2x320x64x64_f32": lambda t: _case_groupnorm(t, 2, 320, 64, 64, t.float32),
    "gn_nhwc_2x320x64x64_bf16": lambda t: _case_groupnorm_nhwc(t, 2, 320, 64, 64, t.bfloat16),
    "gn_nhwc_2x1280x16x16_bf16": lambda t: _case_groupnorm_nhwc(t, 2, 1280, 16, 16, t.bfloat16),
    "q8_0_4608x3072x3072": lambda t: _case_q8(t, 4608, 3072, 3072),
    "q4_k_4608x3072x3072": lambda t: _case_kquant(t, "Q4K", 4608, 3072, 3072),
    "q2_k_4608x3072x3072": lambda t: _case_kquant(t, "Q2K", 4608, 3072, 3072),
    "q3_k_4608x3072x3072": lambda t: _case_kquant(t, "Q3K", 4608, 3072, 3072),
    "q4_k_4608x12288x3072": lambda t: _case_kquant(t, "Q4K", 4608, 12288, 3072),
    "q8_0_4608x12288x3072": lambda t: _case_q8(t, 4608, 12288, 3072),
    "fp8_8192x13824x5120": lambda t: _case_fp8(t, 8192, 13824, 5120),
    # the Wan block's widest GEMMs at 75,600 tokens: fused q/k/v and the feed-forward down
    "fp8_75600x15360x5120": lambda t: _case_fp8(t, 75600, 15360, 5120),
    "fp8_75600x5120x13824": lambda t: _case_fp8(t, 75600, 5120, 13824),
}


def run_case(args):
    import torch
    import sketchpad_b200
    sketchpad_b200.load_library()
    peaks, src = load_peaks()
    fn, work, kind = CASES[args.case](torch)
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    if kind == "flop":
        ach, peak, unit = work / ms / 1e9, peaks["bf16_tflops"], "TFLOP/s"
    else:
        ach, peak, unit = work / ms / 1e6, peaks["hbm_gbs"], "GB/s"
    print(json.dumps({"case": args.case, "ms": ms, "achieved": ach, "unit": unit,
                      "frac": ach / peak, "peak": peak, "peak_source": src, "work": work}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="time eager steps, no CUDA graph")
    ap.add_argument("--no-ulysses", action="store_true",
                    help="N > 1: skip the sequence-parallel Wan block and CFG-split lines")
    ap.add_argument("--case", default=None, choices=sorted(CASES),
                    help="run one kernel workload only (for ncu captures); prints its timing")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.case:
        return run_case(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
