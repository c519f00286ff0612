"""Seeded synthetic inputs: splitmix64 -> Box-Muller (double) -> float32.

One generator shared by the tests, the bench and the parity checks so the
CUDA path and the CPU oracle always see identical inputs. Seeds follow
`0x51580000 + config * 0x100 + layer`.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def seed_for(config: int, layer: int = 0) -> int:
    return 0x51580000 + config * 0x100 + layer


def splitmix64(seed: int, n: int) -> np.ndarray:
    """The first n outputs of splitmix64 started at `seed` (vectorised)."""
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + _GOLDEN * np.arange(1, n + 1, dtype=np.uint64)
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def normal(seed: int, shape, scale: float = 1.0) -> np.ndarray:
    """N(0,1)*scale as float32; pairs of uniforms -> Box-Muller in double."""
    n = int(np.prod(shape))
    m = (n + 1) // 2
    u = splitmix64(seed, 2 * m)
    u1 = ((u[0::2] >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)  # (0, 1]
    u2 = (u[1::2] >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)          # [0, 1)
    r = np.sqrt(-2.0 * np.log(u1))
    t = 2.0 * np.pi * u2
    out = np.empty(2 * m, np.float64)
    out[0::2] = r * np.cos(t)
    out[1::2] = r * np.sin(t)
    return (out[:n] * scale).astype(np.float32).reshape(shape)


def uniform_int(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """n integers uniform in [lo, hi] (inclusive)."""
    u = splitmix64(seed, n)
    return (lo + (u % np.uint64(hi - lo + 1)).astype(np.int64)).astype(np.int64)


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bits, round to nearest even (NaN kept quiet)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    nan = (u & np.uint32(0x7FFFFFFF)) > np.uint32(0x7F800000)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    return np.where(nan, ((u >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16), r)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def to_f16_bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, np.float32).astype(np.float16).view(np.uint16)
