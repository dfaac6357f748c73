"""Communicator of the tensor-parallel exchange: the mllm_comm_* entry points of the C ABI.

One process per GPU.  A `Communicator` is a non-blocking NCCL communicator with the library's
watchdog (include/mllm_attn.h): a collective that runs past `timeout_s`, or an asynchronous NCCL
error, aborts it, after which every call raises `MllmError` with MLLM_ERR_COMM_TIMEOUT or
MLLM_ERR_COMM.  The reference has no counterpart: it runs every layer on one device
(QwenRunner.cpp:236,328), and this carries the o_proj sum (Attention.h:322-325) that sharding
attention by KV-head group adds.
"""
from __future__ import annotations

import ctypes as C

from . import abi

COMM_ID_BYTES = 128
MLLM_ERR_COMM = 8
MLLM_ERR_COMM_TIMEOUT = 9


def unique_id() -> bytes:
    """A fresh communicator id (made on one rank, handed to all)."""
    buf = (C.c_ubyte * COMM_ID_BYTES)()
    abi.call("mllm_comm_unique_id", buf)
    return bytes(buf)


class Communicator:
    """`world` ranks, this one `rank`, on torch's current CUDA device."""

    def __init__(self, rank: int, world: int, uid: bytes, timeout_s: float = 30.0):
        import torch
        if len(uid) != COMM_ID_BYTES:
            raise ValueError("Communicator: the id must be 128 bytes")
        self.rank, self.world, self.timeout_s = rank, world, timeout_s
        self.device = torch.device("cuda", torch.cuda.current_device())
        h = C.c_void_p()
        buf = (C.c_ubyte * COMM_ID_BYTES).from_buffer_copy(uid)
        abi.call("mllm_comm_init", buf, world, rank, float(timeout_s), C.byref(h))
        self.handle = h.value

    @classmethod
    def from_process_group(cls, group=None, timeout_s: float = 30.0) -> "Communicator":
        """Collective over a torch.distributed group (any backend): rank 0 makes the id and the
        group broadcasts it."""
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        box = [unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0,
                                   group=group)
        return cls(rank, world, box[0], timeout_s)

    def _stream(self, stream):
        return abi.stream_handle(stream)

    def all_reduce(self, t, stream=None):
        """In-place bf16 sum over the ranks, enqueued on `stream` (torch's current by default)."""
        import torch
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.device != self.device:
            raise ValueError("Communicator.all_reduce: contiguous bf16 on the communicator's device")
        abi.call("mllm_comm_all_reduce_bf16", self.handle, t.data_ptr(), t.data_ptr(), t.numel(),
                 self._stream(stream))
        return t

    def all_gather(self, src, out, stream=None):
        """out = the ranks' `src` concatenated in rank order (bf16, contiguous)."""
        import torch
        for x in (src, out):
            if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.device != self.device:
                raise ValueError("Communicator.all_gather: contiguous bf16 on the communicator's device")
        if out.numel() != src.numel() * self.world:
            raise ValueError("Communicator.all_gather: out must hold world x src elements")
        abi.call("mllm_comm_all_gather_bf16", self.handle, src.data_ptr(), out.data_ptr(), src.numel(),
                 self._stream(stream))
        return out

    def status(self) -> int:
        """MLLM_OK (0) while healthy; MLLM_ERR_COMM / MLLM_ERR_COMM_TIMEOUT once aborted."""
        return abi.load().mllm_comm_status(self.handle)

    def in_flight(self) -> int:
        return abi.load().mllm_comm_in_flight(self.handle)

    def abort(self) -> None:
        abi.call("mllm_comm_abort", self.handle)

    def close(self) -> None:
        if self.handle is not None:
            h, self.handle = self.handle, None
            abi.call("mllm_comm_destroy", h)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
