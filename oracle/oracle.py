"""CPU oracle bindings -- TEST INFRASTRUCTURE ONLY.

numpy wrappers over oracle/_build/libvxo.so, the plain-C restatement of the
reference's CPU arithmetic (MangoByteLabs/vortex, Rust). Only tests/,
__graft_entry__.smoke() and bench.py's CPU baseline / reference arm use this
module, as the reference to compare against; the product (vortex_b200) never
imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libvxo.so")
_lib = None

INT8, INT4, INT2 = 0, 1, 2
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q8_0 = 0, 1, 2, 3, 8

_P = ctypes.c_void_p
_SZ = ctypes.c_size_t


def build():
    """Compile the oracle library with make (gcc only)."""
    subprocess.check_call(["make", "-s", "-C", _HERE])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        sig = {
            "vxo_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
            "vxo_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "vxo_f32_to_bf16": (ctypes.c_uint16, [ctypes.c_float]),
            "vxo_bf16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
            "vxo_calibrate_minmax": (ctypes.c_double, [_P, _SZ]),
            "vxo_calibrate_minmax_range": (ctypes.c_double, [_P, _SZ, ctypes.c_double, ctypes.c_double]),
            "vxo_pack_int4": (None, [_P, _SZ, _P]),
            "vxo_unpack_int4": (None, [_P, _SZ, _P]),
            "vxo_pack_int2": (None, [_P, _SZ, _P]),
            "vxo_unpack_int2": (None, [_P, _SZ, _P]),
            "vxo_quantize": (_SZ, [_P, _SZ, ctypes.c_int, _SZ, _P, _P, _P]),
            "vxo_num_groups": (_SZ, [_SZ, _SZ]),
            "vxo_dequantize": (None, [_P, _SZ, _SZ, ctypes.c_int, _SZ, _P, _P, _P]),
            "vxo_get_scale": (ctypes.c_double, [_P, _SZ, ctypes.c_int]),
            "vxo_matmul_int": (None, [_P, _P, ctypes.c_int, _SZ, _SZ, _SZ, ctypes.c_double,
                                      ctypes.c_double, ctypes.c_int64, ctypes.c_int64, _P]),
            "vxo_matmul_f64": (None, [_P, _P, _SZ, _SZ, _SZ, _P]),
            "vxo_dequantize_q4_0": (None, [_P, _SZ, _P]),
            "vxo_dequantize_q4_1": (None, [_P, _SZ, _P]),
            "vxo_dequantize_q8_0": (None, [_P, _SZ, _P]),
            "vxo_dequantize_f16": (_SZ, [_P, _SZ, _SZ, _P]),
            "vxo_copy_f32": (_SZ, [_P, _SZ, _SZ, _P]),
            "vxo_ggml_data_size": (_SZ, [ctypes.c_int, _SZ]),
            "vxo_quantize_q8_0": (None, [_P, _SZ, _P]),
            "vxo_quantize_q4_0": (None, [_P, _SZ, _P]),
            "vxo_gemv_blocks": (None, [ctypes.c_int, _P, _SZ, _SZ, _P, _SZ, _P]),
            "vxo_flash_auto_tile": (ctypes.c_int, [_SZ, _SZ]),
            "vxo_flash_attention_forward": (None, [_P, _P, _P, _SZ, _SZ, _SZ, _SZ, ctypes.c_int, _P, _P, _P]),
            "vxo_standard_attention": (None, [_P, _P, _P, _SZ, _SZ, ctypes.c_int, _P]),
            "vxo_flash_attention_backward": (None, [_P, _P, _P, _P, _P, _P, _SZ, _SZ, _SZ, _SZ, ctypes.c_int, _P, _P,
                                                    _P]),
            "vxo_multi_head_flash_attention": (None, [_P, _P, _P, _SZ, _SZ, _SZ, ctypes.c_int, _P]),
            "vxo_attention_rows": (None, [_P, _P, _P, _SZ, _SZ, ctypes.c_int, _P, _SZ, _P, _P]),
            "vxo_paged_attention": (None, [_P, _P, _P, _SZ, _SZ, _P]),
            "vxo_rmsnorm_bias": (None, [_P, _P, _P, _SZ, ctypes.c_double, _P]),
            "vxo_rope_embed": (None, [_P, _SZ, ctypes.c_int64, ctypes.c_int64, _P]),
            "vxo_rope_builtin": (None, [_P, _SZ, _P, _SZ, _P]),
            "vxo_vec_add": (None, [_P, _P, _SZ, _P]),
            "vxo_silu": (ctypes.c_double, [ctypes.c_double]),
            "vxo_vx_exp": (ctypes.c_double, [ctypes.c_double]),
            "vxo_argmax": (ctypes.c_int64, [_P, _SZ]),
            "vxo_lcg_uniform": (ctypes.c_double, [ctypes.c_int64]),
            "vxo_sample_top_p": (ctypes.c_int64, [_P, _SZ, ctypes.c_double, ctypes.c_double, ctypes.c_int64]),
            "vxo_matvec": (None, [_P, _P, _SZ, _SZ, _P]),
            "vxo_tf_param_count": (_SZ, [_P]),
            "vxo_tf_init": (None, [_P, ctypes.c_uint64, _P]),
            "vxo_tf_pos_encoding": (None, [_SZ, _SZ, _P]),
            "vxo_tf_linear": (None, [_P, _SZ, _P, _P, _SZ, _SZ, _P]),
            "vxo_tf_layernorm": (None, [_P, _SZ, _SZ, _P, _P, ctypes.c_float, _P]),
            "vxo_tf_gelu": (None, [_P, _SZ, _P]),
            "vxo_tf_softmax_rows": (None, [_P, _SZ, _SZ, _P]),
            "vxo_tf_forward": (None, [_P, _P, _P, _SZ, _P, _P]),
            "vxo_int8_dot": (ctypes.c_int32, [_P, _P, _SZ]),
            "vxo_int4_dot": (ctypes.c_int32, [_P, _P, _SZ]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def _f64(a):
    return np.ascontiguousarray(a, dtype=np.float64)


# ---- scalar conversions (src/tensor_engine.rs:42-103) ----
def f32_to_f16(x: float) -> int:
    return lib().vxo_f32_to_f16(float(np.float32(x)))


def f16_to_f32(h: int) -> float:
    return lib().vxo_f16_to_f32(int(h))


def f32_to_bf16(x: float) -> int:
    return lib().vxo_f32_to_bf16(float(np.float32(x)))


def bf16_to_f32(b: int) -> float:
    return lib().vxo_bf16_to_f32(int(b))


def f16_bits_to_f32_array(h: np.ndarray) -> np.ndarray:
    """Reference f16 decode applied elementwise (quirky subnormals included)."""
    L = lib()
    h = np.asarray(h, dtype=np.uint16).ravel()
    return np.array([L.vxo_f16_to_f32(int(v)) for v in h], dtype=np.float32)


def f32_array_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Vectorised restatement of tensor_engine::f32_to_bf16 (RNE via bias)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    bias = 0x7FFF + ((u >> 16) & 1)
    return (((u + bias) & 0xFFFFFFFF) >> 16).astype(np.uint16)


def bf16_bits_to_f32_array(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- calibration / packing / quantize ----
def calibrate_minmax(data) -> float:
    d = _f64(data)
    return lib().vxo_calibrate_minmax(_p(d), d.size)


def calibrate_minmax_range(data, qmin, qmax) -> float:
    d = _f64(data)
    return lib().vxo_calibrate_minmax_range(_p(d), d.size, float(qmin), float(qmax))


def pack_int4(values) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.int8)
    out = np.zeros((v.size + 1) // 2, dtype=np.uint8)
    lib().vxo_pack_int4(_p(v), v.size, _p(out))
    return out


def unpack_int4(packed) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.zeros(2 * p.size, dtype=np.int8)
    lib().vxo_unpack_int4(_p(p), p.size, _p(out))
    return out


def pack_int2(values) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.int8)
    out = np.zeros((v.size + 3) // 4, dtype=np.uint8)
    lib().vxo_pack_int2(_p(v), v.size, _p(out))
    return out


def unpack_int2(packed) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.zeros(4 * p.size, dtype=np.int8)
    lib().vxo_unpack_int2(_p(p), p.size, _p(out))
    return out


def quantize(data, fmt: int, group_size: int | None):
    """QuantTensor::quantize -> (packed bytes, scales, zero_points)."""
    d = _f64(data).ravel()
    gs = int(group_size or 0)
    L = lib()
    ng = L.vxo_num_groups(d.size, gs)
    packed = np.zeros(max(d.size, 1), dtype=np.uint8)
    scales = np.zeros(max(ng, 1), dtype=np.float64)
    zps = np.zeros(max(ng, 1), dtype=np.int64)
    nb = L.vxo_quantize(_p(d), d.size, fmt, gs, _p(packed), _p(scales), _p(zps))
    return packed[:nb].copy(), scales[:max(ng, 1)].copy(), zps[:max(ng, 1)].copy()


def dequantize(packed, numel: int, fmt: int, group_size: int | None, scales, zps) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    s = _f64(scales)
    z = np.ascontiguousarray(zps, dtype=np.int64)
    out = np.zeros(max(numel, 1), dtype=np.float64)
    lib().vxo_dequantize(_p(p), p.size, numel, fmt, int(group_size or 0), _p(s), _p(z), _p(out))
    return out[:numel]


def get_scale(scales, per_group: bool) -> float:
    s = _f64(scales)
    return lib().vxo_get_scale(_p(s), s.size, int(per_group))


def matmul_int(a_packed, b_packed, fmt, m, k, n, a_scale, b_scale, a_zp=0, b_zp=0) -> np.ndarray:
    a = np.ascontiguousarray(a_packed, dtype=np.uint8)
    b = np.ascontiguousarray(b_packed, dtype=np.uint8)
    out = np.zeros(m * n, dtype=np.float64)
    lib().vxo_matmul_int(_p(a), _p(b), fmt, m, k, n, a_scale, b_scale, a_zp, b_zp, _p(out))
    return out


def matmul_f64(a, b, m, k, n) -> np.ndarray:
    a = _f64(a)
    b = _f64(b)
    out = np.zeros(m * n, dtype=np.float64)
    lib().vxo_matmul_f64(_p(a), _p(b), m, k, n, _p(out))
    return out


# ---- GGUF blocks ----
def ggml_data_size(t: int, n: int) -> int:
    return lib().vxo_ggml_data_size(t, n)


def _u8(data) -> np.ndarray:
    if isinstance(data, (bytes, bytearray, memoryview)):
        return np.frombuffer(bytes(data), dtype=np.uint8).copy()
    return np.ascontiguousarray(data, dtype=np.uint8)


def dequantize_blocks(t: int, data, n: int) -> np.ndarray:
    d = _u8(data)
    out = np.zeros(max(n, 1), dtype=np.float32)
    L = lib()
    if t == GGML_Q4_0:
        L.vxo_dequantize_q4_0(_p(d), n, _p(out))
    elif t == GGML_Q4_1:
        L.vxo_dequantize_q4_1(_p(d), n, _p(out))
    elif t == GGML_Q8_0:
        L.vxo_dequantize_q8_0(_p(d), n, _p(out))
    elif t == GGML_F16:
        m = L.vxo_dequantize_f16(_p(d), d.size, n, _p(out))
        return out[:m]
    elif t == GGML_F32:
        m = L.vxo_copy_f32(_p(d), d.size, n, _p(out))
        return out[:m]
    else:
        raise ValueError(f"unsupported type {t}")
    return out[:n]


def quantize_blocks(t: int, w) -> np.ndarray:
    """Composed Q8_0/Q4_0 block quantizer over the flat buffer."""
    d = _f64(w).ravel()
    out = np.zeros(max(ggml_data_size(t, d.size), 1), dtype=np.uint8)
    if t == GGML_Q8_0:
        lib().vxo_quantize_q8_0(_p(d), d.size, _p(out))
    elif t == GGML_Q4_0:
        lib().vxo_quantize_q4_0(_p(d), d.size, _p(out))
    else:
        raise ValueError(t)
    return out[:ggml_data_size(t, d.size)]


def gemv_blocks(t: int, blocks, N: int, K: int, x) -> np.ndarray:
    """y[b, r] = sum_k deq(W)[r, k] * x[b, k] in f64; x is [B, K]."""
    bl = np.ascontiguousarray(blocks, dtype=np.uint8)
    xx = _f64(x).reshape(-1, K)
    y = np.zeros((xx.shape[0], N), dtype=np.float64)
    lib().vxo_gemv_blocks(t, _p(bl), N, K, _p(xx), xx.shape[0], _p(y))
    return y


# ---- attention ----
def flash_auto_tile(seq_len: int, head_dim: int) -> int:
    return lib().vxo_flash_auto_tile(seq_len, head_dim)


def flash_attention_forward(q, k, v, d: int, br: int, bc: int, causal: bool):
    q, k, v = _f64(q), _f64(k), _f64(v)
    n = q.size // d
    out = np.zeros(n * d)
    lse = np.zeros(max(n, 1))
    rm = np.zeros(max(n, 1))
    lib().vxo_flash_attention_forward(_p(q), _p(k), _p(v), n, d, br, bc, int(causal), _p(out), _p(lse), _p(rm))
    return out, lse[:n], rm[:n]


def standard_attention(q, k, v, d: int, causal: bool) -> np.ndarray:
    q, k, v = _f64(q), _f64(k), _f64(v)
    n = q.size // d
    out = np.zeros(n * d)
    lib().vxo_standard_attention(_p(q), _p(k), _p(v), n, d, int(causal), _p(out))
    return out


def multi_head_flash_attention(q, k, v, num_heads: int, head_dim: int, causal: bool) -> np.ndarray:
    q, k, v = _f64(q), _f64(k), _f64(v)
    n = q.size // (num_heads * head_dim)
    out = np.zeros(n * num_heads * head_dim)
    lib().vxo_multi_head_flash_attention(_p(q), _p(k), _p(v), n, num_heads, head_dim, int(causal), _p(out))
    return out


def flash_attention_backward(q, k, v, out, grad_out, lse, d: int, br: int, bc: int, causal: bool):
    """flash_attention_backward (src/flash_attention.rs:227-317) of one head:
    inputs [N, d] (flat), lse [N]; returns (grad_q, grad_k, grad_v) flat."""
    q, k, v, out, grad_out, lse = (_f64(t) for t in (q, k, v, out, grad_out, lse))
    n = q.size // d
    gq, gk, gv = (np.zeros(n * d) for _ in range(3))
    lib().vxo_flash_attention_backward(_p(q), _p(k), _p(v), _p(out), _p(grad_out), _p(lse), n, d, br, bc,
                                       int(causal), _p(gq), _p(gk), _p(gv))
    return gq, gk, gv


def attention_rows(q, k, v, d: int, causal: bool, rows):
    """Exact attention of one head ([n, d] inputs) for the listed query rows."""
    q, k, v = _f64(q), _f64(k), _f64(v)
    n = q.size // d
    r = np.ascontiguousarray(rows, dtype=np.int64)
    out = np.zeros((r.size, d))
    lse = np.zeros(max(r.size, 1))
    lib().vxo_attention_rows(_p(q), _p(k), _p(v), n, d, int(causal), _p(r), r.size, _p(out), _p(lse))
    return out, lse[:r.size]


def paged_attention(query, keys, values, head_dim: int) -> np.ndarray:
    q = _f64(query)
    k = _f64(keys).reshape(-1)
    v = _f64(values).reshape(-1)
    ctx = k.size // head_dim
    out = np.zeros(head_dim)
    lib().vxo_paged_attention(_p(q), _p(k), _p(v), ctx, head_dim, _p(out))
    return out


# ---- Llama-style block math ----
def rmsnorm_bias(x, w, b, eps=1e-5) -> np.ndarray:
    x, w, b = _f64(x), _f64(w), _f64(b)
    out = np.zeros(x.size)
    lib().vxo_rmsnorm_bias(_p(x), _p(w), _p(b), x.size, eps, _p(out))
    return out


def rope_embed(x, pos: int, dim: int) -> np.ndarray:
    x = _f64(x)
    out = np.zeros(x.size)
    lib().vxo_rope_embed(_p(x), x.size, int(pos), int(dim), _p(out))
    return out


def rope_builtin(x, freqs) -> np.ndarray:
    x, freqs = _f64(x), _f64(freqs)
    out = np.zeros(x.size)
    lib().vxo_rope_builtin(_p(x), x.size, _p(freqs), freqs.size, _p(out))
    return out


def vec_add(a, b) -> np.ndarray:
    a, b = _f64(a), _f64(b)
    assert a.size == b.size
    out = np.zeros(a.size)
    lib().vxo_vec_add(_p(a), _p(b), a.size, _p(out))
    return out


def silu(x: float) -> float:
    return lib().vxo_silu(float(x))


def matvec(w, v, out_dim: int, in_dim: int) -> np.ndarray:
    w, v = _f64(w), _f64(v)
    out = np.zeros(out_dim)
    lib().vxo_matvec(_p(w), _p(v), out_dim, in_dim, _p(out))
    return out


def int8_dot(a, b) -> int:
    a = np.ascontiguousarray(a, dtype=np.int8)
    b = np.ascontiguousarray(b, dtype=np.int8)
    return lib().vxo_int8_dot(_p(a), _p(b), a.size)


def int4_dot(a, b) -> int:
    a = np.ascontiguousarray(a, dtype=np.uint8)
    b = np.ascontiguousarray(b, dtype=np.uint8)
    return lib().vxo_int4_dot(_p(a), _p(b), a.size)


# ---- f32 GPT-style model (src/transformer.rs:15-841) ----
class TFConfig(ctypes.Structure):
    _fields_ = [("vocab", _SZ), ("d_model", _SZ), ("n_heads", _SZ), ("n_layers", _SZ), ("d_ff", _SZ),
                ("max_seq", _SZ)]


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def tf_config(vocab, d_model, n_heads, n_layers, d_ff, max_seq) -> TFConfig:
    return TFConfig(vocab, d_model, n_heads, n_layers, d_ff, max_seq)


def tf_param_count(cfg: TFConfig) -> int:
    return lib().vxo_tf_param_count(ctypes.byref(cfg))


def tf_init(cfg: TFConfig, seed: int = 42) -> np.ndarray:
    """TransformerModel::new: params in params_vec order."""
    out = np.zeros(tf_param_count(cfg), dtype=np.float32)
    lib().vxo_tf_init(ctypes.byref(cfg), seed, _p(out))
    return out


def tf_pos_encoding(max_len: int, d: int) -> np.ndarray:
    out = np.zeros((max_len, d), dtype=np.float32)
    lib().vxo_tf_pos_encoding(max_len, d, _p(out))
    return out


def tf_linear(x, w, b=None) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    m, k = x.shape
    n = w.shape[0]
    y = np.zeros((m, n), dtype=np.float32)
    bb = _f32(b) if b is not None else None
    lib().vxo_tf_linear(_p(x), m, _p(w), _p(bb) if bb is not None else None, k, n, _p(y))
    return y


def tf_layernorm(x, g, b, eps=1e-5) -> np.ndarray:
    x = _f32(x)
    rows, d = x.shape
    y = np.zeros_like(x)
    lib().vxo_tf_layernorm(_p(x), rows, d, _p(_f32(g)), _p(_f32(b)), eps, _p(y))
    return y


def tf_gelu(x) -> np.ndarray:
    x = _f32(x)
    y = np.zeros_like(x)
    lib().vxo_tf_gelu(_p(x), x.size, _p(y))
    return y


def tf_softmax_rows(x) -> np.ndarray:
    x = _f32(x)
    y = np.zeros_like(x)
    lib().vxo_tf_softmax_rows(_p(x), x.shape[0], x.shape[1], _p(y))
    return y


def tf_forward(cfg: TFConfig, params, tokens, mask=None) -> np.ndarray:
    """TransformerModel::forward: logits [S, vocab] (mask [S, S] or None)."""
    p = _f32(params)
    t = np.ascontiguousarray(tokens, dtype=np.int64)
    S = t.size
    out = np.zeros((S, cfg.vocab), dtype=np.float32)
    m = _f32(mask) if mask is not None else None
    lib().vxo_tf_forward(ctypes.byref(cfg), _p(p), _p(t), S, _p(m) if m is not None else None, _p(out))
    return out


# ---- sampling (stdlib/ai/transformer.vx:36-80, 1163-1260) ----
def vx_exp(x: float) -> float:
    return lib().vxo_vx_exp(float(x))


def argmax(logits) -> int:
    a = _f64(logits)
    return int(lib().vxo_argmax(_p(a), a.size))


def lcg_uniform(seed: int) -> float:
    return lib().vxo_lcg_uniform(int(seed))


def sample_top_p(logits, temperature: float, top_p: float, seed: int) -> int:
    a = _f64(logits)
    return int(lib().vxo_sample_top_p(_p(a), a.size, float(temperature), float(top_p), int(seed)))
