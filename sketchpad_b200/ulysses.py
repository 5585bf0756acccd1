"""Ulysses sequence parallelism: head <-> sequence all-to-all around attention.

The reference has no distributed code (it runs Wan's 75,600-token video DiT on one device,
crates/sketchpad-dit/src/wan.rs:489-573).  Across P GPUs the tokens are sharded
[B, S/P, H, D]; before each attention an all-to-all regroups them as [B, S, H/P, D] (every
rank sees the whole sequence for H/P heads), attention runs locally and unchanged, and a
second all-to-all restores the sequence sharding.  H must divide by P (Wan: 40 heads,
P in {2, 4, 8}); S must divide by P (75,600 does).

Transport: `group` is either this library's NcclComm (sp_ulysses_a2a over its own
non-blocking NCCL communicator, with a host deadline and abort) or a torch.distributed
process group (all_to_all_single: NCCL on GPUs, gloo on CPU for the tests).  Chunk p of the
send buffer goes to rank p, so the pack puts the head group as the leading dimension; the
receive buffer is then every rank's tokens in global token order, which attention reads
through strides without an unpack.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from .comm import NcclComm


def world_size(group) -> int:
    return group.size if isinstance(group, NcclComm) else dist.get_world_size(group)


def rank_of(group) -> int:
    return group.rank if isinstance(group, NcclComm) else dist.get_rank(group)


def _a2a(recv: torch.Tensor, send: torch.Tensor, group) -> None:
    if isinstance(group, NcclComm):
        group.all_to_all(send, recv)
    else:
        dist.all_to_all_single(recv, send, group=group)


def all_gather_tokens(x: torch.Tensor, group) -> torch.Tensor:
    """[B, S/P, ...] per rank -> [B, S, ...] in rank (= global token) order."""
    P = world_size(group)
    xs = x.contiguous()
    buf = torch.empty((P,) + tuple(xs.shape), dtype=xs.dtype, device=xs.device)
    if isinstance(group, NcclComm):
        group.all_gather(xs, buf)
    else:
        dist.all_gather(list(buf.unbind(0)), xs, group=group)
    return buf.movedim(0, 1).reshape(xs.shape[0], P * xs.shape[1], *xs.shape[2:])


def seq_to_head(x: torch.Tensor, group=None) -> torch.Tensor:
    """[B, S/P, H, D] (this rank's tokens, all heads) -> [B, S, H/P, D] (all tokens, this
    rank's head group)."""
    P = world_size(group)
    B, s, H, D = x.shape
    if H % P:
        raise ValueError(f"heads ({H}) must divide by the sequence-parallel size ({P})")
    send = x.reshape(B, s, P, H // P, D).permute(2, 0, 1, 3, 4).contiguous()
    recv = torch.empty_like(send)
    _a2a(recv, send, group)
    # recv[p] = rank p's tokens for this rank's heads (a view when B == 1)
    return recv.permute(1, 0, 2, 3, 4).reshape(B, P * s, H // P, D)


def seq_to_head_qkv(qkv: torch.Tensor, group=None) -> torch.Tensor:
    """The q, k and v of one attention in ONE exchange: [B, S/P, 3, H, D] (the qkv
    projection's output rows) -> [B, S, 3, H/P, D].  One pack copy and one all-to-all
    instead of three of each; for B == 1 the result is the receive buffer itself, and q, k,
    v are its [:, :, j] views (token stride 3*H/P*D)."""
    P = world_size(group)
    B, s, three, H, D = qkv.shape
    if three != 3 or H % P:
        raise ValueError(f"expected [B, s, 3, H, D] with H divisible by {P}")
    send = qkv.reshape(B, s, 3, P, H // P, D).permute(3, 0, 1, 2, 4, 5).contiguous()
    recv = torch.empty_like(send)
    _a2a(recv, send, group)
    return recv.permute(1, 0, 2, 3, 4, 5).reshape(B, P * s, 3, H // P, D)


def head_to_seq(y: torch.Tensor, group=None) -> torch.Tensor:
    """Inverse of seq_to_head: [B, S, H/P, D] -> [B, S/P, H, D]."""
    P = world_size(group)
    B, S, h, D = y.shape
    if S % P:
        raise ValueError(f"sequence ({S}) must divide by the sequence-parallel size ({P})")
    s = S // P
    send = y.reshape(B, P, s, h, D).permute(1, 0, 2, 3, 4).contiguous()
    recv = torch.empty_like(send)
    _a2a(recv, send, group)
    # recv[p] = this rank's tokens for head group p
    return recv.permute(1, 2, 0, 3, 4).reshape(B, s, P * h, D)


def ulysses_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      attn: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor],
                      group=None) -> torch.Tensor:
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


__all__ = ["seq_to_head", "seq_to_head_qkv", "head_to_seq", "ulysses_attention",
           "all_gather_tokens", "a2a_bytes", "world_size", "rank_of"]
