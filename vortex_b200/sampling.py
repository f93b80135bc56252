"""Sampling and continuous batching over libvxb.so: host-side mirror of the
reference's argmax / sample_top_p (stdlib/ai/transformer.vx:1163-1260) and of
ContinuousBatcher with the batcher_* builtins (src/kv_cache.rs:117-154,
255-290). Logits are torch CUDA tensors; the sampling runs on the device.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _native as N
from .quant import _dptr, _stream_ptr, context


def argmax(logits):
    """Greedy token per row (first index of the maximum): f32 [rows, vocab]."""
    import torch
    lg = logits.reshape(-1, logits.shape[-1]).contiguous()
    out = torch.empty(lg.shape[0], dtype=torch.int32, device=lg.device)
    context(lg.device.index).call("vxb_argmax", _dptr(lg), lg.shape[0], lg.shape[1], _dptr(out), _stream_ptr())
    return out


def sample_top_p(logits, temperature: float, top_p: float, seeds):
    """sample_top_p per row of f32 logits [rows, vocab] with one seed per row;
    returns int32 tokens on the device (bit-matched to the reference)."""
    import torch
    lg = logits.reshape(-1, logits.shape[-1]).contiguous().float()
    rows, vocab = lg.shape
    sd = np.ascontiguousarray(np.broadcast_to(np.asarray(seeds, dtype=np.int64), (rows,)))
    out = torch.empty(rows, dtype=torch.int32, device=lg.device)
    context(lg.device.index).call("vxb_sample_top_p", _dptr(lg), rows, vocab, ctypes.c_double(temperature),
                                  ctypes.c_double(top_p), sd.ctypes.data_as(ctypes.c_void_p), _dptr(out),
                                  _stream_ptr())
    return out


class ContinuousBatcher:
    """ContinuousBatcher::new(max_batch_size) (src/kv_cache.rs:128-154)."""

    def __init__(self, max_batch_size: int = 32):
        p = ctypes.c_void_p()
        N.check(N.lib().vxb_batcher_create(int(max_batch_size), ctypes.byref(p)))
        self.ptr = p
        self.max_batch_size = int(max_batch_size)

    def __del__(self):
        try:
            if getattr(self, "ptr", None):
                N.lib().vxb_batcher_destroy(self.ptr)
                self.ptr = None
        except Exception:
            pass

    def add_request(self, tokens) -> int | None:
        """The slot taken, or None when every slot is busy (the batcher_add
        builtin turns that into the error "batcher full")."""
        t = np.ascontiguousarray(tokens, dtype=np.uint64)
        slot = ctypes.c_int(-1)
        rc = N.lib().vxb_batcher_add(self.ptr, t.ctypes.data_as(ctypes.c_void_p), t.size, ctypes.byref(slot))
        if rc == N.VXB_ENOBLOCKS:
            return None
        N.check(rc)
        return slot.value

    def remove_request(self, slot_id: int):
        N.check(N.lib().vxb_batcher_remove(self.ptr, int(slot_id)))

    def num_active(self) -> int:
        n = ctypes.c_int()
        N.check(N.lib().vxb_batcher_num_active(self.ptr, ctypes.byref(n)))
        return n.value

    def slot(self, slot_id: int) -> dict:
        sid, pos, pre, done = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int(), ctypes.c_int()
        nt = ctypes.c_size_t()
        N.check(N.lib().vxb_batcher_slot(self.ptr, int(slot_id), ctypes.byref(sid), ctypes.byref(pos),
                                         ctypes.byref(pre), ctypes.byref(done), ctypes.byref(nt)))
        return {"seq_id": sid.value, "position": pos.value, "is_prefill": bool(pre.value),
                "is_done": bool(done.value), "n_tokens": nt.value}

    def advance(self, slot_id: int, n: int, done: bool = False):
        N.check(N.lib().vxb_batcher_advance(self.ptr, int(slot_id), int(n), int(done)))


def batcher_add(b: ContinuousBatcher, tokens) -> int:
    """The batcher_add builtin (src/kv_cache.rs:260-268): the slot, or the
    error "batcher full"."""
    slot = b.add_request(tokens)
    if slot is None:
        raise N.VxbError(N.VXB_ENOBLOCKS, "batcher full")
    return slot
