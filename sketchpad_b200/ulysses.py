"""Ulysses sequence parallelism: head <-> sequence all-to-all around attention.

The reference has no distributed code (it runs Wan's 75,600-token video DiT on one device,
crates/sketchpad-dit/src/wan.rs:489-573).  Across P GPUs the tokens are sharded
[B, S/P, H, D]; before each attention an all-to-all regroups them as [B, S, H/P, D] (every
rank sees the whole sequence for H/P heads), attention runs locally and unchanged, and a
second all-to-all restores the sequence sharding.  H must divide by P (Wan: 40 heads,
P in {2, 4, 8}); S must divide by P (75,600 does).

Transport: torch.distributed all_to_all_single (NCCL over NVLink on GPUs, gloo on CPU for the
tests).  Chunk p of the send buffer goes to rank p, so the pack puts the head group as the
leading dimension.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def _world(group) -> int:
    return dist.get_world_size(group)


def seq_to_head(x: torch.Tensor, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """[B, S/P, H, D] (this rank's tokens, all heads) -> [B, S, H/P, D] (all tokens, this
    rank's head group)."""
    P = _world(group)
    B, s, H, D = x.shape
    if H % P:
        raise ValueError(f"heads ({H}) must divide by the sequence-parallel size ({P})")
    send = x.reshape(B, s, P, H // P, D).permute(2, 0, 1, 3, 4).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # recv[p] = rank p's tokens for this rank's heads
    return recv.permute(1, 0, 2, 3, 4).reshape(B, P * s, H // P, D)


def head_to_seq(y: torch.Tensor, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """Inverse of seq_to_head: [B, S, H/P, D] -> [B, S/P, H, D]."""
    P = _world(group)
    B, S, h, D = y.shape
    if S % P:
        raise ValueError(f"sequence ({S}) must divide by the sequence-parallel size ({P})")
    s = S // P
    send = y.reshape(B, P, s, h, D).permute(1, 0, 2, 3, 4).contiguous()
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    # recv[p] = this rank's tokens for head group p
    return recv.permute(1, 2, 0, 3, 4).reshape(B, s, P * h, D)


def ulysses_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      attn: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
                      group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """q, k, v: [B, S/P, H, D] token shards -> attention over the full sequence -> [B, S/P, H, D].

    `attn(q, k, v)` takes [B, heads, S, D] views and returns [B, heads, S, D] (e.g.
    sketchpad_b200.flash_attention)."""
    qh, kh, vh = (seq_to_head(t, group) for t in (q, k, v))
    o = attn(qh.transpose(1, 2), kh.transpose(1, 2), vh.transpose(1, 2))
    return head_to_seq(o.transpose(1, 2).contiguous(), group)


def a2a_bytes(B: int, S: int, H: int, D: int, P: int, elem: int = 2) -> int:
    """Bytes one rank sends in one all-to-all of a [B, S, H, D] tensor (the (P-1)/P share
    that leaves the GPU)."""
    return B * (S // P) * H * D * elem * (P - 1) // P


__all__ = ["seq_to_head", "head_to_seq", "ulysses_attention", "a2a_bytes"]
