"""Single ops of the Llama-style block over libvxb.so: host-side mirror of
stdlib/ai/transformer.vx's layer_norm (413-439), rope_embed (442-466),
the SwiGLU gate of feed_forward (591-603), _vec_add (353-366) and of the
`rope` builtin (src/interpreter.rs:2368-2373). Inputs are torch CUDA tensors;
every op runs on the device (the decoder runs the same math fused into its
own kernels). Arguments are checked here before any device call (CPU tensors,
wrong dtypes and undersized outputs raise); a missing libvxb.so raises
VxbError.
"""
from __future__ import annotations

import numpy as np

from .quant import _dptr, _stream_ptr, context


def _cuda_f32(t, what: str):
    import torch
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{what}: a CUDA tensor is expected")
    if t.dtype != torch.float32:
        raise TypeError(f"{what}: f32 expected, got {t.dtype}")
    return t.contiguous()


def _rows(x, what: str):
    x = _cuda_f32(x, what)
    return x.reshape(-1, x.shape[-1]) if x.dim() > 0 else x.reshape(1, 1)


def _out_like(out, ref, what: str):
    """out: None (allocate) or a contiguous f32 CUDA tensor on ref's device
    with at least ref's elements."""
    import torch
    if out is None:
        return torch.empty_like(ref)
    o = _cuda_f32(out, what)
    if o.data_ptr() != out.data_ptr():
        raise ValueError(f"{what}: out must be contiguous")
    if o.device != ref.device or o.numel() < ref.numel():
        raise ValueError(f"{what}: out must hold {ref.numel()} f32 on {ref.device}")
    return o


def layer_norm(x, weight, bias, eps: float = 1e-5):
    """x * weight / sqrt(mean(x^2) + eps) + bias per row of f32 x; bf16 out."""
    import torch
    xr = _rows(x, "layer_norm")
    w, b = _cuda_f32(weight, "layer_norm weight"), _cuda_f32(bias, "layer_norm bias")
    if w.numel() != xr.shape[1] or b.numel() != xr.shape[1]:
        raise ValueError("layer_norm: weight and bias need one value per column")
    out = torch.empty(xr.shape, dtype=torch.bfloat16, device=xr.device)
    context(xr.device.index).call("vxb_rmsnorm", _dptr(xr), _dptr(w), _dptr(b), xr.shape[0], xr.shape[1],
                                  float(eps), _dptr(out), _stream_ptr())
    return out.reshape(x.shape)


def rope_embed(x, pos, dim: int, out=None):
    """Adjacent pairs of each f32 row rotated by pos / 10000^(pair/dim);
    pos is one position or one per row. out may be x (in place)."""
    import torch
    xr = _rows(x, "rope_embed")
    p = np.broadcast_to(np.asarray(pos, dtype=np.int64), (xr.shape[0],)).copy()
    o = _out_like(out, xr, "rope_embed")
    pd = torch.from_numpy(p).to(xr.device)
    context(xr.device.index).call("vxb_rope", _dptr(xr), xr.shape[0], xr.shape[1], _dptr(pd), int(dim), _dptr(o),
                                  _stream_ptr())
    return o.reshape(x.shape)


def rope(x, freqs, out=None):
    """The `rope` builtin: pair i turned by freqs[i] (0 past the list)."""
    import torch
    xr = _rows(x, "rope")
    f = np.ascontiguousarray(np.asarray(freqs, dtype=np.float64).ravel())
    o = _out_like(out, xr, "rope")
    fd = torch.from_numpy(f).to(xr.device)
    context(xr.device.index).call("vxb_rope_angles", _dptr(xr), xr.shape[0], xr.shape[1],
                                  _dptr(fd) if fd.numel() else None, int(fd.numel()), _dptr(o), _stream_ptr())
    return o.reshape(x.shape)


def swiglu(gu):
    """bf16(silu(g) * u) for gu = [g | u] f32 [rows, 2*ffn]."""
    import torch
    g = _rows(gu, "swiglu")
    if g.shape[1] % 2:
        raise ValueError("swiglu: rows of [g | u] need an even length")
    ffn = g.shape[1] // 2
    out = torch.empty((g.shape[0], ffn), dtype=torch.bfloat16, device=g.device)
    context(g.device.index).call("vxb_swiglu", _dptr(g), g.shape[0], ffn, _dptr(out), _stream_ptr())
    return out


def vec_add(a, b, out=None):
    """Residual add a + b (f32, same number of elements); out may be a or b."""
    a, b = _cuda_f32(a, "vec_add"), _cuda_f32(b, "vec_add")
    if a.numel() != b.numel() or a.device != b.device:
        raise ValueError("vec_add: two f32 tensors of one size on one device expected")
    o = _out_like(out, a, "vec_add")
    context(a.device.index).call("vxb_add", _dptr(a), _dptr(b), a.numel(), _dptr(o), _stream_ptr())
    return o
