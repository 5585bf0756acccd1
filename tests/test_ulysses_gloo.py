"""Ulysses all-to-all layout logic on CPU ranks (gloo, world size 2 and 4): sequence-sharded
attention through seq_to_head / head_to_seq equals full-sequence attention computed by the
oracle on one rank (crates/sketchpad-dit/src/wan.rs:351-402 runs it unsharded)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_attn(q, k, v):
    import oracle
    out = oracle.attention(q.numpy(), k.numpy(), v.numpy())
    return torch.from_numpy(out)


def _worker(rank, ws, port, B, S, H, D, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        from sketchpad_b200.ulysses import head_to_seq, seq_to_head, ulysses_attention
        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(B, S, H, D, generator=g) for _ in range(3))
        s = S // ws
        sl = slice(rank * s, (rank + 1) * s)
        # round trip is the identity
        x = q[:, sl].contiguous()
        assert torch.equal(head_to_seq(seq_to_head(x)), x)
        # head-sharded view holds all tokens of this rank's heads
        hg = H // ws
        assert torch.equal(seq_to_head(x), q[:, :, rank * hg:(rank + 1) * hg])
        out = ulysses_attention(q[:, sl].contiguous(), k[:, sl].contiguous(), v[:, sl].contiguous(),
                                _oracle_attn)
        ref = _oracle_attn(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
        np.save(os.path.join(result_dir, f"err{rank}.npy"),
                np.array([float((out - ref[:, sl]).abs().max())]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ws", [2, 4])
def test_ulysses_matches_unsharded_attention(ws, tmp_path):
    B, S, H, D = 1, 64, 8, 16
    mp.spawn(_worker, args=(ws, _free_port(), B, S, H, D, str(tmp_path)), nprocs=ws, join=True)
    errs = [float(np.load(tmp_path / f"err{r}.npy")[0]) for r in range(ws)]
    assert max(errs) < 1e-5


def test_ulysses_rejects_indivisible_heads():
    mp.spawn(_bad_heads, args=(2, _free_port()), nprocs=2, join=True)


def _bad_heads(rank, ws, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        from sketchpad_b200.ulysses import seq_to_head
        try:
            seq_to_head(torch.zeros(1, 4, 3, 8))
        except ValueError:
            return
        raise AssertionError("indivisible heads were accepted")
    finally:
        dist.destroy_process_group()
