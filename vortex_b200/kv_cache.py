"""Paged KV cache and decode attention: host-side mirror of the reference's
PagedKVCache / paged_attention interface (src/kv_cache.rs:29-112) over
libvxb.so. Keys/values live in HBM; queries and outputs are torch CUDA tensors.
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

from . import _native as N
from .quant import _dptr, _stream_ptr, context

BF16 = N.BF16
I8 = N.I8


class PagedKVCache:
    """PagedKVCache::new(num_layers, num_heads, head_dim, block_size, max_blocks)
    (src/kv_cache.rs:41-45); num_heads are the KV heads of a token."""

    def __init__(self, num_layers: int, num_heads: int, head_dim: int, block_size: int = 16,
                 max_blocks: int = 256, max_seqs: int = 64, max_blocks_per_seq: int | None = None,
                 kv_dtype: int = BF16, device=None):
        self.ctx = context(device)
        self.num_layers, self.num_heads, self.head_dim = num_layers, num_heads, head_dim
        self.block_size, self.max_blocks = block_size, max_blocks
        self.kv_dtype = kv_dtype
        mbps = max_blocks_per_seq or max_blocks
        p = ctypes.c_void_p()
        N.check(N.lib().vxb_kv_create(self.ctx.ptr, num_layers, num_heads, head_dim, block_size, max_blocks,
                                      max_seqs, mbps, kv_dtype, ctypes.byref(p)), self.ctx.ptr)
        self.ptr = p

    def __del__(self):
        try:
            if getattr(self, "ptr", None):
                N.lib().vxb_kv_destroy(self.ptr)
                self.ptr = None
        except Exception:
            pass

    def _check(self, rc):
        if rc != N.VXB_OK:
            raise N.VxbError(rc, N.last_error(self.ctx.ptr))

    def append_kv(self, layer: int, seq_ids, k, v):
        """One token per listed sequence: k, v bf16 [n, H, D] on the device."""
        ids = np.ascontiguousarray(np.atleast_1d(seq_ids), dtype=np.int64)
        k = k.contiguous()
        v = v.contiguous()
        self._check(N.lib().vxb_kv_append(self.ptr, layer, ids.size, ids.ctypes.data_as(ctypes.c_void_p),
                                          _dptr(k), _dptr(v), _stream_ptr()))

    def append_seq(self, layer: int, seq_id: int, k, v):
        """Many tokens of one sequence: k, v bf16 [T, H, D]."""
        k = k.contiguous()
        v = v.contiguous()
        T = k.shape[0]
        self._check(N.lib().vxb_kv_append_seq(self.ptr, layer, int(seq_id), T, _dptr(k), _dptr(v), _stream_ptr()))

    def get_kv(self, layer: int, seq_id: int):
        """PagedKVCache::get_kv: (keys, values) as f32 [len, H, D] tensors."""
        import torch
        n = self.seq_len(layer, seq_id)
        k = torch.empty((n, self.num_heads, self.head_dim), dtype=torch.float32, device="cuda")
        v = torch.empty_like(k)
        if n:
            self._check(N.lib().vxb_kv_gather(self.ptr, layer, int(seq_id), _dptr(k), _dptr(v), _stream_ptr()))
        return k, v

    def free_seq(self, seq_id: int):
        self._check(N.lib().vxb_kv_free_seq(self.ptr, int(seq_id)))

    def fork(self, src_seq: int, dst_seq: int, n_tokens: int):
        """Prefix reuse: dst_seq starts as the first n_tokens tokens of
        src_seq (full blocks shared, a partial last block copied)."""
        self._check(N.lib().vxb_kv_fork(self.ptr, int(src_seq), int(dst_seq), int(n_tokens), _stream_ptr()))

    def stats(self) -> dict:
        out = (ctypes.c_int64 * 6)()
        self._check(N.lib().vxb_kv_stats(self.ptr, out))
        return {"used_blocks": out[0], "free_blocks": out[1], "block_size": out[2], "num_seqs": out[3],
                "device_bytes": out[4], "sequences": out[5]}

    def used_blocks(self) -> int:
        return self.stats()["used_blocks"]

    def free_block_count(self) -> int:
        return self.stats()["free_blocks"]

    def seq_len(self, layer: int, seq_id: int) -> int:
        n = ctypes.c_int64()
        self._check(N.lib().vxb_kv_seq_len(self.ptr, layer, int(seq_id), ctypes.byref(n)))
        return n.value

    def block_table(self, layer: int, seq_id: int) -> list[int]:
        n = ctypes.c_int()
        self._check(N.lib().vxb_kv_block_table(self.ptr, layer, int(seq_id), None, 0, ctypes.byref(n)))
        buf = (ctypes.c_int32 * max(n.value, 1))()
        self._check(N.lib().vxb_kv_block_table(self.ptr, layer, int(seq_id), buf, n.value, ctypes.byref(n)))
        return list(buf[:n.value])

    def attention(self, layer: int, seq_ids, q, softmax_scale: float | None = None, out=None, lse=None):
        """paged_attention for one new query per sequence: q bf16 [n, Hq, D]
        -> bf16 [n, Hq, D] (and the natural-log sum-exp if lse is given)."""
        import torch
        ids = np.ascontiguousarray(np.atleast_1d(seq_ids), dtype=np.int64)
        q = q.contiguous()
        Hq = q.shape[1]
        if out is None:
            out = torch.empty_like(q)
        scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(self.head_dim)
        self._check(N.lib().vxb_decode_attention(self.ptr, layer, ids.size, ids.ctypes.data_as(ctypes.c_void_p),
                                                 _dptr(q), Hq, ctypes.c_float(scale), _dptr(out),
                                                 _dptr(lse) if lse is not None else None, _stream_ptr()))
        return out
