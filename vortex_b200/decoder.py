"""Llama-style quantized decoder over libvxb.so (host-side mirror of the
transformer forward / generate interface, stdlib/ai/transformer.vx:958-1177,
and of the transformer_* builtins' call pattern, src/transformer.rs:940-1034).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _native as N
from .quant import context


class DecoderConfig(ctypes.Structure):
    _fields_ = [("vocab_size", ctypes.c_int), ("dim", ctypes.c_int), ("n_layers", ctypes.c_int),
                ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int), ("ffn_dim", ctypes.c_int),
                ("max_batch", ctypes.c_int), ("max_seq", ctypes.c_int), ("norm_eps", ctypes.c_float),
                ("weight_fmt", ctypes.c_int), ("kv_dtype", ctypes.c_int), ("kv_block_size", ctypes.c_int)]


LLAMA_7B = dict(vocab_size=32000, dim=4096, n_layers=32, n_heads=32, n_kv_heads=32, ffn_dim=11008,
                norm_eps=1e-5, weight_fmt=N.Q4_0, kv_dtype=N.BF16, kv_block_size=16)

# weight slots of vxb_decoder_set_weight
WQ, WK, WV, WO, W1, W2, W3, LN1_W, LN1_B, LN2_W, LN2_B = range(11)
EMBED, FINAL_W, FINAL_B, OUTPUT = range(4)


class Decoder:
    """comm (optional): a vortex_b200.comm.Comm; the decoder is then this
    rank's tensor-parallel part, and every rank makes the same calls."""

    def __init__(self, max_batch: int, max_seq: int, device=None, comm=None, **cfg):
        self.ctx = comm.ctx if comm is not None else context(device)
        L = N.lib()
        c = dict(LLAMA_7B)
        c.update(cfg)
        self.cfg = DecoderConfig(**{k: c[k] for k, _ in DecoderConfig._fields_ if k in c},
                                 max_batch=max_batch, max_seq=max_seq)
        p = ctypes.c_void_p()
        if comm is None:
            N.check(L.vxb_decoder_create(self.ctx.ptr, ctypes.addressof(self.cfg), ctypes.byref(p)), self.ctx.ptr)
        else:
            N.check(L.vxb_decoder_create_tp(self.ctx.ptr, ctypes.addressof(self.cfg), comm.ptr, ctypes.byref(p)),
                    self.ctx.ptr)
        self.comm = comm
        self.ptr = p
        self.vocab = self.cfg.vocab_size

    def close(self):
        if getattr(self, "ptr", None):
            N.lib().vxb_decoder_destroy(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        if rc != N.VXB_OK:
            raise N.VxbError(rc, N.last_error(self.ctx.ptr))

    def init_random(self, seed: int = 42, sigma: float = 0.02):
        self._check(N.lib().vxb_decoder_init_random(self.ptr, seed, sigma))

    def set_weight(self, layer: int, which: int, data: np.ndarray):
        a = np.ascontiguousarray(data)
        self._check(N.lib().vxb_decoder_set_weight(self.ptr, layer, which, a.ctypes.data_as(ctypes.c_void_p),
                                                   a.nbytes))

    def step(self, seq_ids, tokens, want_logits: bool = False):
        ids = np.ascontiguousarray(seq_ids, dtype=np.int64)
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = np.zeros(ids.size, dtype=np.int32)
        logits = np.zeros((ids.size, self.vocab), dtype=np.float32) if want_logits else None
        self._check(N.lib().vxb_decoder_step(self.ptr, ids.size, ids.ctypes.data_as(ctypes.c_void_p),
                                             tok.ctypes.data_as(ctypes.c_void_p), nxt.ctypes.data_as(ctypes.c_void_p),
                                             logits.ctypes.data_as(ctypes.c_void_p) if want_logits else None))
        return (nxt, logits) if want_logits else nxt

    def prefill(self, seq_id: int, tokens, want_logits: bool = False):
        """Whole prompt of a new sequence in one pass (K2 GEMM + K3 flash
        attention); returns the greedy next token (and the last logits)."""
        tok = np.ascontiguousarray(tokens, dtype=np.int32)
        nxt = np.zeros(1, dtype=np.int32)
        logits = np.zeros(self.vocab, dtype=np.float32) if want_logits else None
        self._check(N.lib().vxb_decoder_prefill(self.ptr, int(seq_id), tok.ctypes.data_as(ctypes.c_void_p), tok.size,
                                                nxt.ctypes.data_as(ctypes.c_void_p),
                                                logits.ctypes.data_as(ctypes.c_void_p) if want_logits else None))
        return (int(nxt[0]), logits) if want_logits else int(nxt[0])

    def step_device(self, seq_ids, d_tokens, d_next, stream=None):
        import torch
        ids = np.ascontiguousarray(seq_ids, dtype=np.int64)
        s = stream if stream is not None else torch.cuda.current_stream()
        self._check(N.lib().vxb_decoder_step_device(self.ptr, ids.size, ids.ctypes.data_as(ctypes.c_void_p),
                                                    ctypes.c_void_p(d_tokens.data_ptr()),
                                                    ctypes.c_void_p(d_next.data_ptr()) if d_next is not None else None,
                                                    ctypes.c_void_p(s.cuda_stream)))

    def free_seq(self, seq_id: int):
        self._check(N.lib().vxb_decoder_free_seq(self.ptr, int(seq_id)))

    def stream_handle(self) -> int:
        p = ctypes.c_void_p()
        self._check(N.lib().vxb_decoder_stream(self.ptr, ctypes.byref(p)))
        return p.value or 0
