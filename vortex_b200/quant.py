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


class BlockRows:
    """A weight matrix W [N, K] kept on the device as its GGUF rows (any of
    F32, F16, Q4_0, Q4_1, Q8_0: row n = the blocks of W[n, :]), e.g. a Q4_1
    projection from a GGUF file (gguf_loader.rs:413-531)."""

    def __init__(self, data, ggml_type: int, n_rows: int, k_cols: int):
        self.data = data
        self.type = int(ggml_type)
        self.N, self.K = int(n_rows), int(k_cols)
        self.device = data.device
        self.ctx = context(data.device.index)
        if data.numel() < N.lib().vxb_block_bytes(self.type, self.N * self.K):
            raise N.VxbError(N.VXB_EINVAL, "BlockRows: buffer too short")

    def dequantize(self):
        torch = _torch()
        out = torch.empty(self.N * self.K, dtype=torch.float32, device=self.device)
        self.ctx.call("vxb_dequantize_blocks", self.type, _dptr(self.data), self.N * self.K, _dptr(out),
                      _stream_ptr())
        return out.reshape(self.N, self.K)

    def gemv(self, x, out=None, out_dtype=None):
        """y = x @ deq(W)^T for bf16 x [B, K]."""
        torch = _torch()
        x = x.contiguous()
        B = x.numel() // self.K
        dt = out_dtype or (out.dtype if out is not None else torch.float32)
        if out is None:
            out = torch.empty((B, self.N), dtype=dt, device=x.device)
        self.ctx.call("vxb_gemv_blocks", self.type, _dptr(self.data), self.N, self.K, _dptr(x), B,
                      N.F32 if dt == torch.float32 else N.BF16, _dptr(out), _stream_ptr())
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


# ---------------------------------------------------------------- QuantTensor (mean-scale int matmul)

QT_INT8 = 0
QT_INT4 = 1
_QT_FORMATS = {"INT8": QT_INT8, "INT4": QT_INT4}


class QuantTensor:
    """Mirror of QuantTensor (src/quantize.rs:70-94) for the INT8 and INT4
    formats: codes (`data`), shape, and a PerTensor (group_size None) or
    PerGroup scheme with f64 scales and zero points. quantize / dequantize run
    on the host (the reference's rules); matmul runs on the device
    (vxb_quant_matmul, bit-exact with QuantTensor::matmul)."""

    def __init__(self, data, shape, fmt, scales, zero_points, group_size=None):
        self.data = np.ascontiguousarray(data, dtype=np.uint8)
        self.shape = tuple(int(s) for s in shape)
        self.fmt = _QT_FORMATS[fmt.upper()] if isinstance(fmt, str) else int(fmt)
        if self.fmt not in (QT_INT8, QT_INT4):
            raise N.VxbError(N.VXB_EINVAL, f"QuantTensor: format {fmt} (INT8 or INT4)")
        self.scales = np.ascontiguousarray(scales, dtype=np.float64)
        self.zero_points = np.ascontiguousarray(zero_points, dtype=np.int64)
        self.group_size = group_size

    @property
    def numel(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    @classmethod
    def quantize(cls, data, shape, fmt, group_size=None):
        """QuantTensor::quantize (src/quantize.rs:81-163) for INT8 / INT4."""
        f = _QT_FORMATS[fmt.upper()] if isinstance(fmt, str) else int(fmt)
        a = np.ascontiguousarray(data, dtype=np.float64).ravel()
        if a.size != int(np.prod(shape)):
            raise N.VxbError(N.VXB_EINVAL, "quantize: data length must match shape product")
        gs = int(group_size) if group_size else 0
        L = N.lib()
        packed = np.zeros(max(L.vxb_qt_data_bytes(f, a.size), 1), dtype=np.uint8)
        ng = max(L.vxb_qt_num_groups(a.size, gs), 1)
        scales = np.zeros(ng, dtype=np.float64)
        zps = np.zeros(ng, dtype=np.int64)
        N.check(L.vxb_qt_quantize(f, _ptr(a), a.size, gs, _ptr(packed), _ptr(scales), _ptr(zps)))
        nb = L.vxb_qt_data_bytes(f, a.size)
        ng = L.vxb_qt_num_groups(a.size, gs)
        return cls(packed[:nb], shape, f, scales[:max(ng, 1)], zps[:max(ng, 1)], gs or None)

    def codes(self) -> np.ndarray:
        """The signed codes (unpack_int4 for INT4, src/quantize.rs:675-687)."""
        if self.fmt == QT_INT8:
            return self.data.view(np.int8).astype(np.int64)
        lo = (self.data & 0xF).astype(np.int64)
        hi = (self.data >> 4).astype(np.int64)
        q = np.stack([lo, hi], axis=1).ravel()
        return (q ^ 8) - 8

    def dequantize(self) -> np.ndarray:
        """QuantTensor::dequantize for INT8 / INT4 (src/quantize.rs:325-370):
        (q - zp) as f64 * scale per element of its group."""
        q = self.codes()[:self.numel]
        if self.group_size is None:
            return (q - int(self.zero_points[0])).astype(np.float64) * float(self.scales[0])
        g = np.arange(q.size) // self.group_size
        return (q - self.zero_points[g]).astype(np.float64) * self.scales[g]

    def get_scale(self) -> float:
        """get_scale (src/quantize.rs:534-545): the scale, or the mean of the
        group scales."""
        if self.group_size is None:
            return float(self.scales[0])
        out = ctypes.c_double()
        s = self.scales
        N.check(N.lib().vxb_qt_mean_scale(_ptr(s), s.size, ctypes.byref(out)))
        return out.value

    def get_zero_point(self) -> int:
        return int(self.zero_points[0]) if self.group_size is None else 0

    def matmul(self, other: "QuantTensor", device=None) -> np.ndarray:
        """QuantTensor::matmul for INT8 x INT8 / INT4 x INT4 (src/quantize.rs:
        447-515) on the device: f64 [m * n]."""
        torch = _torch()
        if len(self.shape) != 2 or len(other.shape) != 2 or self.shape[1] != other.shape[0]:
            raise N.VxbError(N.VXB_EINVAL, "matmul: shapes must be [m, k] x [k, n]")
        if self.fmt != other.fmt:
            raise N.VxbError(N.VXB_EUNSUPPORTED, "matmul: mixed formats take the dequantize fallback")
        m, k = self.shape
        n = other.shape[1]
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else int(device))
        a = torch.from_numpy(self.data).to(dev)
        b = torch.from_numpy(other.data).to(dev)
        out = torch.empty(m * n, dtype=torch.float64, device=dev)
        context(dev.index).call("vxb_quant_matmul", self.fmt, _dptr(a), _dptr(b), m, k, n,
                                ctypes.c_double(self.get_scale()), ctypes.c_double(other.get_scale()),
                                self.get_zero_point(), other.get_zero_point(), _dptr(out), _stream_ptr())
        return out.cpu().numpy()
