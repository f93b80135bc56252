"""Quantized weights and the decode GEMV: host-side mirror of the reference's
QuantTensor / weight_only_matmul interface (src/quantize.rs:70-94, 845-852)
and of the GGUF block codec (src/gguf_loader.rs:413-498), over libvxb.so.

Host arrays are numpy; device tensors are torch CUDA tensors (torch is used for
device memory and streams only -- all arithmetic runs in libvxb.so).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _native as N

Q4_0 = N.Q4_0
Q8_0 = N.Q8_0
FORMATS = {"Q4_0": Q4_0, "Q8_0": Q8_0, "INT4": Q4_0, "INT8": Q8_0}


def _fmt(fmt) -> int:
    if isinstance(fmt, str):
        try:
            return FORMATS[fmt.upper()]
        except KeyError:
            raise N.VxbError(N.VXB_EINVAL, f"unknown format '{fmt}'")
    return int(fmt)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def block_bytes(fmt, n: int) -> int:
    return N.lib().vxb_block_bytes(_fmt(fmt), n)


def pack_blocks(fmt, w) -> np.ndarray:
    """f32/f64 weights (flat, any shape) -> GGUF blocks, bit-exact with the
    reference rules (QuantTensor::quantize PerGroup, group 32; f16 scales)."""
    f = _fmt(fmt)
    a = np.asarray(w)
    out = np.zeros(max(block_bytes(f, a.size), 1), dtype=np.uint8)
    if a.dtype == np.float32:
        a = np.ascontiguousarray(a).ravel()
        N.check(N.lib().vxb_pack_blocks_f32(f, _ptr(a), a.size, _ptr(out)))
    else:
        a = np.ascontiguousarray(a, dtype=np.float64).ravel()
        N.check(N.lib().vxb_pack_blocks_f64(f, _ptr(a), a.size, _ptr(out)))
    return out[:block_bytes(f, a.size)]


def unpack_blocks(fmt, blocks, n: int) -> np.ndarray:
    """GGUF blocks -> f32 values (dequantize_q4_0 / dequantize_q8_0)."""
    f = _fmt(fmt)
    b = np.ascontiguousarray(np.frombuffer(bytes(blocks), dtype=np.uint8) if isinstance(blocks, (bytes, bytearray))
                             else blocks, dtype=np.uint8)
    if b.size < block_bytes(f, n):
        raise N.VxbError(N.VXB_EINVAL, "unpack_blocks: block buffer too short")
    out = np.zeros(max(n, 1), dtype=np.float32)
    N.check(N.lib().vxb_unpack_blocks(f, _ptr(b), n, _ptr(out)))
    return out[:n]


# ---------------------------------------------------------------- device side

def _torch():
    import torch
    return torch


def _stream_ptr(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _dptr(t):
    return ctypes.c_void_p(t.data_ptr())


def context(device=None) -> N.Context:
    torch = _torch()
    dev = torch.cuda.current_device() if device is None else int(device)
    return N.Context.get(dev)


def quantize_blocks(w, fmt):
    """Device quantizer: f32 CUDA tensor -> uint8 CUDA tensor of GGUF blocks."""
    torch = _torch()
    f = _fmt(fmt)
    w = w.contiguous()
    if w.dtype != torch.float32 or not w.is_cuda:
        raise N.VxbError(N.VXB_EINVAL, "quantize_blocks expects a float32 CUDA tensor")
    out = torch.empty(block_bytes(f, w.numel()), dtype=torch.uint8, device=w.device)
    ctx = context(w.device.index)
    ctx.call("vxb_quantize_blocks", f, _dptr(w), w.numel(), _dptr(out), _stream_ptr())
    return out


def dequantize_blocks(blocks, fmt, n: int):
    torch = _torch()
    f = _fmt(fmt)
    out = torch.empty(n, dtype=torch.float32, device=blocks.device)
    context(blocks.device.index).call("vxb_dequantize_blocks", f, _dptr(blocks), n, _dptr(out), _stream_ptr())
    return out


class TiledWeight:
    """A quantized weight matrix W [N, K] resident in HBM in the kernels'
    tiled layout (lossless regrouping of the GGUF blocks)."""

    def __init__(self, blocks, fmt, n_rows: int, k_cols: int):
        torch = _torch()
        self.fmt = _fmt(fmt)
        self.N = int(n_rows)
        self.K = int(k_cols)
        if self.K % 32:
            raise N.VxbError(N.VXB_EINVAL, "K must be a multiple of 32")
        if blocks.numel() < block_bytes(self.fmt, self.N * self.K):
            raise N.VxbError(N.VXB_EINVAL, "block buffer too short")
        self.device = blocks.device
        nbytes = N.lib().vxb_tiled_bytes(self.fmt, self.N, self.K)
        self.tiled = torch.empty(nbytes, dtype=torch.uint8, device=blocks.device)
        self.ctx = context(blocks.device.index)
        self.ctx.call("vxb_tile_weights", self.fmt, _dptr(blocks), self.N, self.K, _dptr(self.tiled), _stream_ptr())

    @classmethod
    def from_tiled(cls, tiled, fmt, n_rows: int, k_cols: int):
        """Wrap an already tiled device buffer (e.g. from a GGUF upload)."""
        self = cls.__new__(cls)
        self.fmt = _fmt(fmt)
        self.N, self.K = int(n_rows), int(k_cols)
        self.device = tiled.device
        self.tiled = tiled
        self.ctx = context(tiled.device.index)
        return self

    @classmethod
    def from_float(cls, w, fmt):
        """Quantize a float32 CUDA matrix [N, K] on the device and tile it."""
        blocks = quantize_blocks(w.reshape(-1), fmt)
        return cls(blocks, fmt, w.shape[0], w.shape[1])

    def to_blocks(self):
        torch = _torch()
        out = torch.empty(block_bytes(self.fmt, self.N * self.K), dtype=torch.uint8, device=self.device)
        self.ctx.call("vxb_untile_weights", self.fmt, _dptr(self.tiled), self.N, self.K, _dptr(out), _stream_ptr())
        return out

    @property
    def nbytes_blocks(self) -> int:
        return block_bytes(self.fmt, self.N * self.K)

    def gemv(self, x, out=None, out_dtype=None):
        """y = x @ deq(W)^T for x bf16 [B, K] (B <= 32), y f32 or bf16 [B, N]."""
        torch = _torch()
        if x.dtype != torch.bfloat16:
            raise N.VxbError(N.VXB_EINVAL, "gemv expects bf16 activations")
        x = x.contiguous()
        B = x.numel() // self.K
        if x.numel() != B * self.K:
            raise N.VxbError(N.VXB_EINVAL, "activation size is not a multiple of K")
        dt = out_dtype or (out.dtype if out is not None else torch.float32)
        code = N.F32 if dt == torch.float32 else N.BF16
        if out is None:
            out = torch.empty((B, self.N), dtype=dt, device=x.device)
        self.ctx.call("vxb_gemv_q", self.fmt, _dptr(self.tiled), self.N, self.K, _dptr(x), B, code, _dptr(out),
                      _stream_ptr())
        return out


    def gemm(self, x, out=None, out_dtype=None):
        """Y = X @ deq(W)^T for many rows (prefill GEMM on tcgen05): x bf16
        [M, K], y f32 or bf16 [M, N]."""
        torch = _torch()
        if x.dtype != torch.bfloat16:
            raise N.VxbError(N.VXB_EINVAL, "gemm expects bf16 activations")
        x = x.contiguous()
        M = x.numel() // self.K
        if x.numel() != M * self.K:
            raise N.VxbError(N.VXB_EINVAL, "activation size is not a multiple of K")
        dt = out_dtype or (out.dtype if out is not None else torch.float32)
        code = N.F32 if dt == torch.float32 else N.BF16
        if out is None:
            out = torch.empty((M, self.N), dtype=dt, device=x.device)
        self.ctx.call("vxb_gemm_q", self.fmt, _dptr(self.tiled), self.N, self.K, _dptr(x), M, code, _dptr(out),
                      _stream_ptr())
        return out


def weight_only_matmul(w: TiledWeight, activations):
    """Mirror of weight_only_matmul (src/quantize.rs:845-852) for W stored
    [N, K]: returns activations [M, K] @ deq(W)^T as f32 [M, N]: the decode
    GEMV for up to 32 rows, the tcgen05 GEMM above that."""
    torch = _torch()
    x = activations.to(torch.bfloat16).contiguous()
    M = x.shape[0]
    if M > 32:
        return w.gemm(x)
    out = torch.empty((M, w.N), dtype=torch.float32, device=x.device)
    w.gemv(x, out=out)
    return out
