"""Bit-exact conformance of the device's pinned consensus math with the CPU
oracle: exp_f32, rsqrt_f32 and granite_rope_sin_cos, through the C-ABI
qxc_consensus_math_conformance.

The reference runs the same check between its Rust functions and its Metal
kernel on eight inputs (qx-metal/src/lib.rs:15488-15511); the oracle's three
functions are pinned to the reference's own known-answer tests in
test_oracle.py.
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NAN_BITS = 0x7FC00000


def f32_bits(x: float) -> int:
    return int(np.array([x], dtype=np.float32).view(np.uint32)[0])


def position_of(x: np.float32) -> int:
    """Rust's saturating `value as u32` (and PTX cvt.rzi.u32.f32)."""
    if math.isnan(x) or x <= 0:
        return 0
    if x >= 4294967295.0:
        return 0xFFFFFFFF
    return int(math.floor(float(x)))


def expected(oracle, inputs):
    rows = []
    for i, x in enumerate(np.asarray(inputs, dtype=np.float32)):
        e = oracle.exp_f32(float(x)) if math.isfinite(x) else None
        r = oracle.rsqrt_f32(float(x))
        sc = oracle.granite_rope_sin_cos(position_of(x), i % 32)
        rows.append((
            f32_bits(e) if e is not None else NAN_BITS,
            f32_bits(r) if r is not None else NAN_BITS,
            f32_bits(sc[0]) if sc is not None else NAN_BITS,
            f32_bits(sc[1]) if sc is not None else NAN_BITS,
        ))
    return rows


def test_reference_conformance_inputs(gpu_ctx, oracle):
    """The reference's eight inputs (qx-metal/src/lib.rs:15489): every
    function has a value there, and the device bits equal the oracle's."""
    inputs = [1.0e-6, 1.0, 17.0, 128.0, 511.0, 1024.0, 2048.0, 4095.0]
    want = expected(oracle, inputs)
    assert all(NAN_BITS not in row for row in want)
    assert gpu_ctx.run_consensus_math_conformance(inputs) == want


def test_edge_inputs(gpu_ctx, oracle):
    """Inputs where the pinned functions clamp or have no value: zero and
    negatives (no rsqrt), the exp clamps at -87 / 88, non-finite values, and
    positions whose RoPE angle leaves the pinned range (|angle| > 4096)."""
    inputs = [0.0, -0.0, -1.0, -87.5, -87.0, 88.0, 88.5, 1e30, float("inf"), float("-inf"), float("nan"),
              4096.0, 4097.0, 65535.0, 1e6, 3e9, 5e9, 1.17549435e-38, 1e-45, 3.4028235e38]
    want = expected(oracle, inputs)
    assert NAN_BITS in {v for row in want for v in row}
    assert gpu_ctx.run_consensus_math_conformance(inputs) == want


def test_random_sweep(gpu_ctx, oracle):
    """4096 seeded inputs over the attention score domain (exp of negative
    arguments), RMS-norm denominators and RoPE positions up to 8192, so every
    pair index meets many positions."""
    rng = np.random.default_rng(1234)
    inputs = np.concatenate([
        rng.uniform(-90.0, 0.0, 1024),
        np.exp(rng.uniform(-20.0, 20.0, 1024)),
        rng.integers(0, 8192, 2048).astype(np.float32) + rng.uniform(0, 1, 2048),
    ]).astype(np.float32)
    want = expected(oracle, inputs)
    got = gpu_ctx.run_consensus_math_conformance(inputs)
    bad = [(i, float(inputs[i]), got[i], want[i]) for i in range(len(inputs)) if got[i] != want[i]]
    assert not bad, bad[:5]


def test_empty_input(gpu_ctx):
    assert gpu_ctx.run_consensus_math_conformance([]) == []
