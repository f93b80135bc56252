"""Flash-attention forward (K3) over libvxb.so: host-side mirror of the
reference's flash_attention_forward / multi_head_flash_attention
(src/flash_attention.rs:53-159, 519-564).

Tensors are torch CUDA tensors (torch is used for device memory and streams
only; the arithmetic runs in libvxb.so on tcgen05 tensor cores).
"""
from __future__ import annotations

import ctypes
import math

from . import _native as N
from .quant import _dptr, _stream_ptr, context


def flash_attention(q, k, v, causal: bool = True, softmax_scale: float | None = None, out=None, lse=None,
                    stream=None):
    """O = softmax(scale * Q K^T [causal]) V per head.

    q: bf16 [B, S, H, 128]; k, v: bf16 [B, S, Hkv, 128] with Hkv dividing H.
    Returns (out bf16 [B, S, H, 128], lse f32 [B, H, S] natural log)."""
    import torch
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise N.VxbError(N.VXB_EINVAL, "flash_attention: q, k, v must be [B, S, heads, d]")
    B, S, H, d = q.shape
    Hkv = k.shape[2]
    if k.shape != (B, S, Hkv, d) or v.shape != k.shape:
        raise N.VxbError(N.VXB_EINVAL, "flash_attention: k and v must be [B, S, Hkv, d] like q")
    for t in (q, k, v):
        if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
            raise N.VxbError(N.VXB_EINVAL, "flash_attention: tensors must be contiguous bf16 on the GPU")
    scale = 1.0 / math.sqrt(d) if softmax_scale is None else float(softmax_scale)
    if out is None:
        out = torch.empty_like(q)
    if lse is None:
        lse = torch.empty(B, H, S, device=q.device, dtype=torch.float32)
    ctx = context(q.device.index)
    ctx.call("vxb_flash_fwd", _dptr(q), _dptr(k), _dptr(v), B, H, Hkv, S, d, ctypes.c_float(scale), int(causal),
             _dptr(out), _dptr(lse), _stream_ptr(stream))
    return out, lse


def multi_head_flash_attention(q, k, v, num_heads: int, head_dim: int, causal: bool):
    """The reference's multi-head entry: q, k, v are [N, num_heads * head_dim]
    rows with the heads interleaved (src/flash_attention.rs:545-551); returns
    the output in the same layout."""
    n = q.shape[0]
    shp = (1, n, num_heads, head_dim)
    o, _ = flash_attention(q.reshape(shp).contiguous(), k.reshape(shp).contiguous(), v.reshape(shp).contiguous(),
                           causal=causal)
    return o.reshape(n, num_heads * head_dim)


def flash_attention_backward(q, k, v, out, grad_out, lse, causal: bool = True, softmax_scale: float | None = None,
                             stream=None):
    """flash_attention_backward (src/flash_attention.rs:227-317) on the
    device: q / out / grad_out bf16 [B, S, H, 128], k / v bf16 [B, S, Hkv,
    128], lse f32 [B, H, S] (the forward's second output). Returns (dq, dk,
    dv) as f32 tensors of the shapes of q, k, v."""
    import torch
    B, S, H, d = q.shape
    Hkv = k.shape[2]
    for t in (q, k, v, out, grad_out):
        if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
            raise N.VxbError(N.VXB_EINVAL, "flash_attention_backward: tensors must be contiguous bf16 on the GPU")
    if out.shape != q.shape or grad_out.shape != q.shape or v.shape != k.shape:
        raise N.VxbError(N.VXB_EINVAL, "flash_attention_backward: shape mismatch")
    lse = lse.contiguous().float()
    scale = 1.0 / math.sqrt(d) if softmax_scale is None else float(softmax_scale)
    dq = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    dk = torch.empty(k.shape, dtype=torch.float32, device=q.device)
    dv = torch.empty(v.shape, dtype=torch.float32, device=q.device)
    ctx = context(q.device.index)
    ctx.call("vxb_flash_bwd", _dptr(q), _dptr(k), _dptr(v), _dptr(out), _dptr(grad_out), _dptr(lse), B, H, Hkv, S,
             d, ctypes.c_float(scale), int(causal), _dptr(dq), _dptr(dk), _dptr(dv), _stream_ptr(stream))
    return dq, dk, dv
