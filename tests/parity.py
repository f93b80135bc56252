"""Shared parity metrics for the GPU-vs-oracle tests."""
import numpy as np


def rel_err(y, r, floor=1e-3):
    """max_i |y_i - r_i| / max(|r_i|, floor * max_j |r_j|) -- elementwise relative
    error with a floor at 1e-3 of the largest reference magnitude."""
    y = np.asarray(y, dtype=np.float64).ravel()
    r = np.asarray(r, dtype=np.float64).ravel()
    if r.size == 0:
        return 0.0
    den = np.maximum(np.abs(r), floor * np.max(np.abs(r)))
    den[den == 0] = 1.0
    return float(np.max(np.abs(y - r) / den))


def norm_err(y, r):
    """||y - r||_inf / ||r||_inf."""
    y = np.asarray(y, dtype=np.float64).ravel()
    r = np.asarray(r, dtype=np.float64).ravel()
    m = np.max(np.abs(r)) if r.size else 0.0
    return float(np.max(np.abs(y - r)) / (m if m > 0 else 1.0)) if r.size else 0.0


def bf16_round(x):
    """Round f32 values to bf16 (RNE, tensor_engine::f32_to_bf16) and return f32."""
    from oracle import oracle as O
    return O.bf16_bits_to_f32_array(O.f32_array_to_bf16_bits(np.asarray(x, dtype=np.float32)))
