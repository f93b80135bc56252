"""Single ops of the Llama-style block over libvxb.so: host-side mirror of
stdlib/ai/transformer.vx's layer_norm (413-439), rope_embed (442-466),
the SwiGLU gate of feed_forward (591-603), _vec_add (353-366) and of the
`rope` builtin (src/interpreter.rs:2368-2373). Inputs are torch CUDA tensors;
every op runs on the device (the decoder runs the same math fused into its
own kernels). A missing libvxb.so raises VxbError.
"""
from __future__ import annotations

import numpy as np

from .quant import _dptr, _stream_ptr, context


def _rows(x):
    import torch
    x = x.contiguous()
    if x.dtype != torch.float32:
        raise TypeError("f32 input expected")
    return x.reshape(-1, x.shape[-1]) if x.dim() > 0 else x.reshape(1, 1)


def layer_norm(x, weight, bias, eps: float = 1e-5):
    """x * weight / sqrt(mean(x^2) + eps) + bias per row of f32 x; bf16 out."""
    import torch
    xr = _rows(x)
    w, b = weight.contiguous().float(), bias.contiguous().float()
    out = torch.empty(xr.shape, dtype=torch.bfloat16, device=xr.device)
    context(xr.device.index).call("vxb_rmsnorm", _dptr(xr), _dptr(w), _dptr(b), xr.shape[0], xr.shape[1],
                                  float(eps), _dptr(out), _stream_ptr())
    return out.reshape(x.shape)


def rope_embed(x, pos, dim: int, out=None):
    """Adjacent pairs of each f32 row rotated by pos / 10000^(pair/dim);
    pos is one position or one per row. out may be x (in place)."""
    import torch
    xr = _rows(x)
    p = torch.as_tensor(np.broadcast_to(np.asarray(pos, dtype=np.int64), (xr.shape[0],)).copy()).to(xr.device)
    o = torch.empty_like(xr) if out is None else out
    context(xr.device.index).call("vxb_rope", _dptr(xr), xr.shape[0], xr.shape[1], _dptr(p), int(dim), _dptr(o),
                                  _stream_ptr())
    return o.reshape(x.shape)


def rope(x, freqs, out=None):
    """The `rope` builtin: pair i turned by freqs[i] (0 past the list)."""
    import torch
    xr = _rows(x)
    f = torch.as_tensor(np.asarray(freqs, dtype=np.float64)).to(xr.device)
    o = torch.empty_like(xr) if out is None else out
    context(xr.device.index).call("vxb_rope_angles", _dptr(xr), xr.shape[0], xr.shape[1],
                                  _dptr(f) if f.numel() else None, int(f.numel()), _dptr(o), _stream_ptr())
    return o.reshape(x.shape)


def swiglu(gu):
    """bf16(silu(g) * u) for gu = [g | u] f32 [rows, 2*ffn]."""
    import torch
    g = _rows(gu)
    ffn = g.shape[1] // 2
    out = torch.empty((g.shape[0], ffn), dtype=torch.bfloat16, device=g.device)
    context(g.device.index).call("vxb_swiglu", _dptr(g), g.shape[0], ffn, _dptr(out), _stream_ptr())
    return out


def vec_add(a, b, out=None):
    """Residual add a + b (f32, same number of elements); out may be a or b."""
    import torch
    a, b = a.contiguous(), b.contiguous()
    if a.numel() != b.numel() or a.dtype != torch.float32 or b.dtype != torch.float32:
        raise ValueError("vec_add: two f32 tensors of one size expected")
    o = torch.empty_like(a) if out is None else out
    context(a.device.index).call("vxb_add", _dptr(a), _dptr(b), a.numel(), _dptr(o), _stream_ptr())
    return o
