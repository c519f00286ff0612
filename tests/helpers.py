"""Shared helpers for the parity tests (inputs, error metrics)."""
import numpy as np

from qx_b200 import synthetic as syn


def normwise(actual, expected) -> float:
    """max|actual - expected| / max|expected| (the normwise relative error
    the parity gates use; elementwise relative error is ill-conditioned for
    attention outputs near zero)."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    return float(np.max(np.abs(a - e)) / max(np.max(np.abs(e)), 1e-30))


def granite_inputs(seed: int, prefix: int, capacity: int):
    """q[1024], k[512], v[512] and cache rows [prefix][8][64] (f32, N(0,1))."""
    q = syn.normal(seed, (1024,))
    k = syn.normal(seed + 0x10000000, (512,))
    v = syn.normal(seed + 0x20000000, (512,))
    kc = syn.normal(seed + 0x30000000, (prefix, 8, 64))
    vc = syn.normal(seed + 0x40000000, (prefix, 8, 64))
    return q, k, v, kc, vc


def as_kv(x: np.ndarray, dtype: int) -> np.ndarray:
    if dtype == 0:
        return np.ascontiguousarray(x, np.float32)
    if dtype == 1:
        return syn.to_bf16_bits(x)
    return syn.to_f16_bits(x)
