"""The reference's f32 TransformerModel (src/transformer.rs:658-815) on the
GPU: host-side mirror of TransformerConfig / TransformerModel::new /
forward / params_vec / set_params over libvxb.so."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _native as N
from .quant import context


class TModelConfig(ctypes.Structure):
    _fields_ = [("vocab_size", ctypes.c_int), ("d_model", ctypes.c_int), ("n_heads", ctypes.c_int),
                ("n_layers", ctypes.c_int), ("d_ff", ctypes.c_int), ("max_seq_len", ctypes.c_int)]


class TransformerModel:
    """TransformerModel::new(config): Xavier weights from the reference's
    xorshift generator (seed 42); the same parameters bit for bit."""

    def __init__(self, vocab_size: int, d_model: int, n_heads: int, n_layers: int, d_ff: int, max_seq_len: int,
                 device=None):
        self.ctx = context(device)
        self.cfg = TModelConfig(vocab_size, d_model, n_heads, n_layers, d_ff, max_seq_len)
        p = ctypes.c_void_p()
        N.check(N.lib().vxb_tmodel_create(self.ctx.ptr, ctypes.byref(self.cfg), ctypes.byref(p)), self.ctx.ptr)
        self.ptr = p
        n = ctypes.c_size_t()
        N.check(N.lib().vxb_tmodel_param_count(self.ptr, ctypes.byref(n)))
        self.n_params = n.value

    def close(self):
        if getattr(self, "ptr", None):
            N.lib().vxb_tmodel_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def params_vec(self) -> np.ndarray:
        out = np.zeros(self.n_params, dtype=np.float32)
        N.check(N.lib().vxb_tmodel_get_params(self.ptr, out.ctypes.data_as(ctypes.c_void_p), out.size), self.ctx.ptr)
        return out

    def set_params(self, params):
        p = np.ascontiguousarray(params, dtype=np.float32)
        N.check(N.lib().vxb_tmodel_set_params(self.ptr, p.ctypes.data_as(ctypes.c_void_p), p.size), self.ctx.ptr)

    def forward(self, token_ids, mask=None) -> np.ndarray:
        """logits [seq_len, vocab_size]; mask [seq_len, seq_len] (entries < 0.5
        are masked) or None."""
        t = np.ascontiguousarray(token_ids, dtype=np.int32)
        S = t.size
        out = np.zeros((S, self.cfg.vocab_size), dtype=np.float32)
        m = None if mask is None else np.ascontiguousarray(mask, dtype=np.float32).reshape(S, S)
        N.check(N.lib().vxb_tmodel_forward(self.ptr, t.ctypes.data_as(ctypes.c_void_p), S,
                                           m.ctypes.data_as(ctypes.c_void_p) if m is not None else None,
                                           out.ctypes.data_as(ctypes.c_void_p)), self.ctx.ptr)
        return out
