"""NcclComm: the library's own NCCL communicator (sp_nccl_* / sp_ulysses_a2a in
include/sketchpad_b200.h) for the sequence-parallel Wan exchange.

The communicator is non-blocking: every call returns once its work is enqueued, polling
NCCL's asynchronous state against a host deadline; an NCCL error or an expired deadline
aborts the communicator and raises CommError, so a rank that never joins or stops answering
ends the other ranks' calls with an error instead of a hang.  The reference has no
collectives at all (it runs Wan on one device, crates/sketchpad-dit/src/wan.rs:720-757); this
is the transport of the one exchange step splitting it across GPUs needs.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from ._torch import ptr, stream_ptr

NCCL_IN_PROGRESS = 7


class CommError(RuntimeError):
    """An NCCL failure or a passed deadline (status SP_ERR_COMM); the communicator is
    aborted when this is raised by a collective."""


def _dt(t: torch.Tensor) -> int:
    try:
        return {torch.float32: _lib.SP_F32, torch.float16: _lib.SP_F16,
                torch.bfloat16: _lib.SP_BF16}[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}") from None


def _call(name, *args):
    rc = getattr(_lib.load(), name)(*args)
    if rc == -8:
        raise CommError(_lib.load().sp_last_error().decode())
    if rc != 0:
        raise RuntimeError(f"{name}: {_lib.load().sp_last_error().decode()} (status {rc})")


def unique_id() -> bytes:
    """A fresh NCCL unique id (made on the host; share it with the other ranks)."""
    n = _lib.load().sp_nccl_unique_id_bytes()
    buf = ctypes.create_string_buffer(n)
    _call("sp_nccl_unique_id", buf, n)
    return buf.raw


class NcclComm:
    def __init__(self, rank: int, size: int, uid: bytes, device: Optional[torch.device] = None,
                 timeout: float = 60.0):
        """Joins rank `rank` of `size` on `device` (default: the current device); raises
        CommError when the others do not join within `timeout` seconds."""
        self.rank, self.size, self.timeout = rank, size, float(timeout)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else \
            torch.device(device)
        self._comm = ctypes.c_void_p()
        # a list here receives (start, end) CUDA events around every all-to-all (timing)
        self.events = None
        with torch.cuda.device(self.device):
            _call("sp_nccl_comm_init", ctypes.byref(self._comm), size, rank,
                  ctypes.create_string_buffer(uid, len(uid)), self.timeout)

    @classmethod
    def from_group(cls, group=None, timeout: float = 60.0) -> "NcclComm":
        """One communicator over the ranks of a torch.distributed group: rank 0 of the group
        makes the id and the group broadcasts it (a host-side exchange)."""
        import torch.distributed as dist
        rank, size = dist.get_rank(group), dist.get_world_size(group)
        obj = [unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group else 0,
                                   group=group)
        return cls(rank, size, obj[0], timeout=timeout)

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._comm:
            raise CommError("the communicator was destroyed or aborted")
        return self._comm

    def all_to_all(self, send: torch.Tensor, recv: torch.Tensor) -> torch.Tensor:
        """sp_ulysses_a2a: chunk p (numel / size elements) of `send` goes to rank p; chunk p
        of `recv` comes from rank p.  Both contiguous, same dtype and size, on this device."""
        if send.numel() != recv.numel() or send.numel() % self.size or send.dtype != recv.dtype:
            raise ValueError("send and recv must hold the same number (a multiple of the "
                             "communicator size) of elements of one dtype")
        if not (send.is_contiguous() and recv.is_contiguous()):
            raise ValueError("send and recv must be contiguous")
        ev = self.events
        if ev is not None:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
        _call("sp_ulysses_a2a", ptr(send), ptr(recv), send.numel() // self.size, _dt(send),
              self.handle, stream_ptr(send.device), self.timeout)
        if ev is not None:
            b.record()
            ev.append((a, b, send.numel() * send.element_size() * (self.size - 1) // self.size))
        return recv

    def all_gather(self, send: torch.Tensor, recv: torch.Tensor) -> torch.Tensor:
        if recv.numel() != send.numel() * self.size or send.dtype != recv.dtype:
            raise ValueError("recv must hold size x send.numel() elements of send's dtype")
        if not (send.is_contiguous() and recv.is_contiguous()):
            raise ValueError("send and recv must be contiguous")
        _call("sp_nccl_all_gather", ptr(send), ptr(recv), send.numel(), _dt(send), self.handle,
              stream_ptr(send.device), self.timeout)
        return recv

    def wait(self, timeout: Optional[float] = None) -> None:
        """Waits for the current stream while watching the communicator (sp_nccl_wait);
        aborts it and raises CommError on an NCCL error or when the deadline passes."""
        _call("sp_nccl_wait", self.handle, stream_ptr(self.device),
              self.timeout if timeout is None else float(timeout))

    def poll(self) -> int:
        st = ctypes.c_int()
        _call("sp_nccl_comm_poll", self.handle, ctypes.byref(st))
        return st.value

    def abort(self) -> None:
        if self._comm:
            _lib.load().sp_nccl_comm_abort(self._comm)
            self._comm = ctypes.c_void_p()

    def destroy(self) -> None:
        if self._comm:
            c, self._comm = self._comm, ctypes.c_void_p()
            _call("sp_nccl_comm_destroy", c, self.timeout)


__all__ = ["NcclComm", "CommError", "unique_id"]
