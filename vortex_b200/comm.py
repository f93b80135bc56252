"""Tensor-parallel communicator over libvxb.so (NCCL over NVLink / NVSwitch):
the host side of the nccl_ffi.rs externs (src/nccl_ffi.rs:12-72).

One process per GPU. Rank 0 makes a unique id, the caller shares it over its
own channel (here: a torch.distributed process group, e.g. gloo or nccl), and
every rank joins.
"""
from __future__ import annotations

import ctypes

from . import _native as N
from .quant import context

UNIQUE_ID_BYTES = 128


def unique_id() -> bytes:
    buf = ctypes.create_string_buffer(UNIQUE_ID_BYTES)
    N.check(N.lib().vxb_nccl_unique_id(buf))
    return buf.raw


def share_unique_id(rank: int, group=None, make=unique_id) -> bytes:
    """Rank 0 makes the id (make()), every rank of the torch.distributed
    group receives it. Works over any backend (gloo on CPU included)."""
    import torch.distributed as dist
    obj = [make() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != UNIQUE_ID_BYTES:
        raise N.VxbError(N.VXB_EINVAL, "share_unique_id: bad unique id")
    return bytes(uid)


class Comm:
    """vxb_comm_init / vxb_comm_destroy for rank `rank` of `nranks`."""

    def __init__(self, nranks: int, rank: int, uid: bytes, device=None):
        self.ctx = context(device)
        p = ctypes.c_void_p()
        N.check(N.lib().vxb_comm_init(self.ctx.ptr, nranks, rank, ctypes.c_char_p(uid), ctypes.byref(p)),
                self.ctx.ptr)
        self.ptr = p
        self.nranks, self.rank = nranks, rank

    def allreduce_sum(self, t, stream=None):
        """In place over a contiguous f32 or bf16 torch CUDA tensor."""
        import torch
        dt = {torch.float32: N.F32, torch.bfloat16: N.BF16}.get(t.dtype)
        if dt is None or not t.is_contiguous():
            raise N.VxbError(N.VXB_EINVAL, "allreduce_sum: contiguous f32 or bf16 tensor required")
        s = stream if stream is not None else torch.cuda.current_stream()
        N.check(N.lib().vxb_allreduce_sum(self.ptr, ctypes.c_void_p(t.data_ptr()), t.numel(), dt,
                                          ctypes.c_void_p(s.cuda_stream)), self.ctx.ptr)

    def close(self):
        if getattr(self, "ptr", None):
            N.lib().vxb_comm_destroy(self.ptr)
            self.ptr = None
