"""The interpreter builtins of the hot path, over libvxb.so.

Mirror of the reference's builtin adapters for this path - same names, the
same argument order and defaults, the same result shapes and error strings -
with the arithmetic on the device:

  quantize / dequantize / quantized_matmul / compression_ratio
      src/interpreter.rs:7278-7346, value_to_quant_tensor 7348-7389
  flash_attention (builtin_flash_attention, src/interpreter.rs:2216-2265)
  kv_cache_new / _append / _attention / _stats / _free_seq / _memory and
  batcher_new / _add / _active / _remove
      src/kv_cache.rs:183-290

A QuantTensor value is a dict with the fields the reference's struct carries
(format, shape, compression_ratio, _data, _scale, _zero_point); handles are
integers into per-process tables, as the reference's LazyLock<Mutex<Vec<_>>>
tables. Errors raise BuiltinError with the reference's message.
"""
from __future__ import annotations

import math
import threading

import numpy as np

from . import quant as Q


class BuiltinError(RuntimeError):
    """The builtin's Err(String)."""


_QT_BITS = {"INT8": 8, "INT4": 4}


# ---------------------------------------------------------------- quantization

def quantize(*args):
    """quantize(data, shape, format[, group_size]) -> QuantTensor struct."""
    if len(args) < 3:
        raise BuiltinError("quantize requires at least 3 args: data, shape, format")
    data, shape, fmt = args[0], args[1], args[2]
    if not isinstance(data, (list, tuple, np.ndarray)):
        raise BuiltinError("quantize: first arg must be array")
    if not isinstance(shape, (list, tuple)):
        raise BuiltinError("quantize: second arg must be array (shape)")
    if not all(isinstance(s, (int, np.integer)) for s in shape):
        raise BuiltinError("quantize: shape must be array of ints")
    if not isinstance(fmt, str):
        raise BuiltinError("quantize: third arg must be format string")
    if fmt.upper() not in _QT_BITS:
        raise BuiltinError(f"quantize: unknown format '{fmt}'")
    gs = args[3] if len(args) > 3 and isinstance(args[3], (int, np.integer)) and args[3] > 0 else None
    vals = np.asarray(data, dtype=np.float64).ravel()
    if vals.size != int(np.prod(shape)):
        raise BuiltinError("data length must match shape product")
    qt = Q.QuantTensor.quantize(vals, shape, fmt.upper(), gs)
    return {"format": fmt, "shape": [int(s) for s in shape],
            "compression_ratio": 32.0 / _QT_BITS[fmt.upper()],
            "_data": [int(b) for b in qt.data], "_scale": qt.get_scale(), "_zero_point": qt.get_zero_point()}


def _value_to_quant_tensor(v) -> Q.QuantTensor:
    """value_to_quant_tensor: a PerTensor tensor with the struct's mean
    _scale (1.0 if absent) and _zero_point (0 if absent)."""
    if not isinstance(v, dict):
        raise BuiltinError("expected QuantTensor struct")
    fmt = v.get("format")
    if not isinstance(fmt, str):
        raise BuiltinError("QuantTensor missing format field")
    if fmt.upper() not in _QT_BITS:
        raise BuiltinError(f"unknown format '{fmt}'")
    if "shape" not in v:
        raise BuiltinError("QuantTensor missing shape")
    if "_data" not in v:
        raise BuiltinError("QuantTensor missing _data")
    scale = v.get("_scale")
    scale = float(scale) if isinstance(scale, float) else 1.0
    zp = v.get("_zero_point")
    zp = int(zp) if isinstance(zp, (int, np.integer)) else 0
    data = np.asarray([int(b) & 0xFF for b in v["_data"]], dtype=np.uint8)
    return Q.QuantTensor(data, v["shape"], fmt.upper(), [scale], [zp], None)


def dequantize(*args):
    """dequantize(qtensor) -> array (with the struct's single mean scale)."""
    if not args:
        raise BuiltinError("dequantize requires 1 arg: qtensor")
    return [float(x) for x in _value_to_quant_tensor(args[0]).dequantize()]


def quantized_matmul(*args):
    """quantized_matmul(a_q, b_q) -> flat array [m * n] (device, bit-exact)."""
    if len(args) < 2:
        raise BuiltinError("quantized_matmul requires 2 args: a_q, b_q")
    a = _value_to_quant_tensor(args[0])
    b = _value_to_quant_tensor(args[1])
    if len(a.shape) != 2 or len(b.shape) != 2 or a.shape[1] != b.shape[0]:
        raise BuiltinError("quantized_matmul: shapes must be [m, k] x [k, n]")
    if a.fmt != b.fmt:
        # the reference dequantizes both and multiplies in f64 (src/quantize.rs:463-468)
        m, k = a.shape
        n = b.shape[1]
        return [float(x) for x in (a.dequantize().reshape(m, k) @ b.dequantize().reshape(k, n)).ravel()]
    return [float(x) for x in a.matmul(b)]


def compression_ratio(*args):
    if not args:
        raise BuiltinError("compression_ratio requires 1 arg: qtensor")
    qt = _value_to_quant_tensor(args[0])
    return 32.0 / (8 if qt.fmt == Q.QT_INT8 else 4)


# ---------------------------------------------------------------- flash attention

def flash_attention(*args):
    """flash_attention(q, k, v, [num_heads], [causal]) -> [N][H*d] (the
    builtin_flash_attention adapter: 2-D [N, H*d] rows, heads interleaved).
    The device kernel takes head_dim 128."""
    import torch

    from . import attention as A
    if len(args) < 3:
        raise BuiltinError("flash_attention expects (q, k, v, [num_heads], [causal])")
    mats = [np.asarray(a, dtype=np.float64) for a in args[:3]]
    if any(m.size == 0 for m in mats):
        return []
    n, total = mats[0].shape
    heads = args[3] if len(args) > 3 and isinstance(args[3], (int, np.integer)) else 1
    causal = args[4] if len(args) > 4 and isinstance(args[4], bool) else False
    hd = total // heads
    if hd * heads != total:
        raise BuiltinError(f"flash_attention: dim {total} not divisible by {heads} heads")
    q, k, v = (torch.from_numpy(m.astype(np.float32)).cuda().to(torch.bfloat16) for m in mats)
    o = A.multi_head_flash_attention(q, k, v, heads, hd, causal)
    return o.float().cpu().numpy().astype(np.float64).tolist()


def flash_attention_backward(*args):
    """flash_attention_backward(q, k, v, output, grad_output, [num_heads],
    [causal]) -> (grad_q, grad_k, grad_v) as [N][H*d] (the
    builtin_flash_attention_backward adapter, src/interpreter.rs:2267-2340:
    per head, lse from a non-causal forward and a non-causal backward - the
    adapter reads `causal` but never uses it)."""
    import torch

    from . import attention as A
    if len(args) < 5:
        raise BuiltinError("flash_attention_backward expects (q, k, v, output, grad_output, [num_heads], [causal])")
    mats = [np.asarray(a, dtype=np.float64) for a in args[:5]]
    if mats[0].size == 0:
        return ([], [], [])
    n, total = mats[0].shape
    heads = args[5] if len(args) > 5 and isinstance(args[5], (int, np.integer)) else 1
    hd = total // heads
    q, k, v, o, do = (torch.from_numpy(m.astype(np.float32)).cuda().to(torch.bfloat16).reshape(1, n, heads, hd)
                      for m in mats)
    _, lse = A.flash_attention(q, k, v, causal=False)
    dq, dk, dv = A.flash_attention_backward(q, k, v, o, do, lse, causal=False)
    return tuple(t.reshape(n, total).cpu().numpy().astype(np.float64).tolist() for t in (dq, dk, dv))


# ---------------------------------------------------------------- KV cache and batcher

_LOCK = threading.Lock()
_CACHES: list = []
_BATCHERS: list = []


class _OneHeadCache:
    """A kv_cache_new cache. The reference's cache is head-agnostic (each
    appended key / value is one head_dim vector), so the device cache holds
    one KV head (num_heads is kept for the record, as the reference does).
    The block accounting the builtins report (stats, memory, the out-of-blocks
    error) is the reference's own, kept here per (layer, seq_id) table:
    a table takes ceil(len / block_size) of max_blocks blocks, a table entry
    exists from its first append attempt on (src/kv_cache.rs:54-67). The
    device pages hold 16 tokens (a multiple of 16 at least block_size), so
    max_blocks device pages always suffice."""

    def __init__(self, nl, nh, hd, bs, mb):
        from . import kv_cache as KV
        if nl < 1 or bs < 1 or mb < 0:
            raise BuiltinError("kv_cache_new: num_layers, block_size and max_blocks must be positive")
        self.num_layers, self.num_heads, self.head_dim, self.block_size, self.max_blocks = nl, nh, hd, bs, mb
        self.tables = {}  # (layer, seq) -> tokens
        dev_bs = 16 * -(-bs // 16)
        self.cache = KV.PagedKVCache(nl, 1, hd, dev_bs, max_blocks=max(mb, 1), max_seqs=max(64, mb),
                                     max_blocks_per_seq=max(mb, 1))

    def used_blocks(self):
        return sum(-(-n // self.block_size) for n in self.tables.values())


def _int_arg(args, i, default=None, err=None):
    v = args[i] if len(args) > i else None
    if isinstance(v, (int, np.integer)) and not isinstance(v, bool):
        return int(v)
    if err is not None:
        raise BuiltinError(err)
    return default


def kv_cache_new(*args):
    """kv_cache_new([num_layers=12], [num_heads=8], [head_dim=64],
    [block_size=16], [max_blocks=256]) -> cache id."""
    nl, nh, hd = _int_arg(args, 0, 12), _int_arg(args, 1, 8), _int_arg(args, 2, 64)
    bs, mb = _int_arg(args, 3, 16), _int_arg(args, 4, 256)
    c = _OneHeadCache(nl, nh, hd, bs, mb)
    with _LOCK:
        _CACHES.append(c)
        return len(_CACHES) - 1


def _cache(cid):
    with _LOCK:
        if not 0 <= cid < len(_CACHES) or _CACHES[cid] is None:
            raise BuiltinError("invalid cache")
        return _CACHES[cid]


def _floats(v, what):
    if v is None:
        raise BuiltinError(f"need {what}")
    if not isinstance(v, (list, tuple, np.ndarray)):
        raise BuiltinError("expected array")
    return np.asarray(v, dtype=np.float64).ravel()


def kv_cache_append(*args):
    """kv_cache_append(cache_id, layer, seq_id, key, value) -> true."""
    import torch
    cid = _int_arg(args, 0, err="need cache_id")
    layer = _int_arg(args, 1, err="need layer")
    seq = _int_arg(args, 2, err="need seq_id")
    key = _floats(args[3] if len(args) > 3 else None, "key")
    value = _floats(args[4] if len(args) > 4 else None, "value")
    c = _cache(cid)
    if key.size != c.head_dim or value.size != c.head_dim:
        raise BuiltinError(f"kv_cache_append: key and value must hold head_dim = {c.head_dim} values")
    if not 0 <= layer < c.num_layers:
        raise BuiltinError(f"kv_cache_append: layer {layer} out of range")
    n = c.tables.setdefault((layer, seq), 0)
    if n % c.block_size == 0 and c.used_blocks() >= c.max_blocks:
        raise BuiltinError("KV cache out of blocks")
    k = torch.from_numpy(key.astype(np.float32)).cuda().to(torch.bfloat16).reshape(1, 1, -1)
    v = torch.from_numpy(value.astype(np.float32)).cuda().to(torch.bfloat16).reshape(1, 1, -1)
    c.cache.append_kv(layer, [seq], k, v)
    c.tables[(layer, seq)] = n + 1
    return True


def kv_cache_attention(*args):
    """kv_cache_attention(cache_id, query, layer, seq_id) -> [head_dim]:
    paged_attention over every cached token of the sequence, scale
    1/sqrt(head_dim); zeros for an empty sequence."""
    import torch
    cid = _int_arg(args, 0, err="need cache_id")
    query = _floats(args[1] if len(args) > 1 else None, "query")
    layer = _int_arg(args, 2, err="need layer")
    seq = _int_arg(args, 3, err="need seq_id")
    c = _cache(cid)
    if query.size != c.head_dim:
        raise BuiltinError(f"kv_cache_attention: query must hold head_dim = {c.head_dim} values")
    q = torch.from_numpy(query.astype(np.float32)).cuda().to(torch.bfloat16).reshape(1, 1, -1)
    out = c.cache.attention(layer, [seq], q, softmax_scale=1.0 / math.sqrt(c.head_dim))
    return out.float().cpu().numpy().ravel().astype(np.float64).tolist()


def kv_cache_stats(*args):
    """kv_cache_stats(cache_id) -> KVCacheStats {used_blocks, free_blocks,
    block_size, num_seqs} (num_seqs = block tables, one per (layer, seq))."""
    cid = _int_arg(args, 0, err="need cache_id")
    c = _cache(cid)
    used = c.used_blocks()
    return {"used_blocks": used, "free_blocks": c.max_blocks - used, "block_size": c.block_size,
            "num_seqs": len(c.tables)}


def kv_cache_free_seq(*args):
    cid = _int_arg(args, 0, err="need cache_id")
    seq = _int_arg(args, 1, err="need seq_id")
    c = _cache(cid)
    c.tables = {key: n for key, n in c.tables.items() if key[1] != seq}
    c.cache.free_seq(seq)
    return True


def kv_cache_memory(*args):
    """kv_cache_memory(cache_id) -> bytes the reference's f64 cache would
    hold: used_blocks * block_size * head_dim * 2 * 8."""
    cid = _int_arg(args, 0, err="need cache_id")
    c = _cache(cid)
    return c.used_blocks() * c.block_size * c.head_dim * 2 * 8


def batcher_new(*args):
    from .sampling import ContinuousBatcher
    b = ContinuousBatcher(_int_arg(args, 0, 32))
    with _LOCK:
        _BATCHERS.append(b)
        return len(_BATCHERS) - 1


def _batcher(bid):
    with _LOCK:
        if not 0 <= bid < len(_BATCHERS):
            raise BuiltinError("invalid batcher")
        return _BATCHERS[bid]


def batcher_add(*args):
    """batcher_add(batcher_id, tokens) -> slot, or "batcher full"."""
    bid = _int_arg(args, 0, err="need batcher_id")
    toks = args[1] if len(args) > 1 and isinstance(args[1], (list, tuple)) else []
    toks = [int(t) if isinstance(t, (int, np.integer)) else 0 for t in toks]
    slot = _batcher(bid).add_request(toks)
    if slot is None:
        raise BuiltinError("batcher full")
    return slot


def batcher_active(*args):
    return _batcher(_int_arg(args, 0, err="need batcher_id")).num_active()


def batcher_remove(*args):
    bid = _int_arg(args, 0, err="need batcher_id")
    slot = _int_arg(args, 1, err="need slot_id")
    _batcher(bid).remove_request(slot)
    return True
