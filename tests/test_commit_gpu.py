"""KV-slot and residual-checkpoint commitments on the GPU against the oracle.

The reference hashes KV slots and residual snapshots with BLAKE3 Merkle trees
for its verification protocol (kernels/verification_hash.metal; CPU
definitions qx-commit state.rs:213-257, :334-368; golden case qx-metal
lib.rs:15531-15604). Gate: every digest byte-identical to the oracle's.
"""
import numpy as np
import pytest

from qx_b200 import (BF16, F16, F32, HASH_PER_CHUNK, HASH_PER_SLOT, MODEL_GRANITE, MODEL_QWEN3, KvArena,
                     QxError)
from qx_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def filled_arena(ctx, model, layers, tokens, kd, vd, seed, seq=0, sequences=1, cap=None):
    """An arena whose first `tokens` rows of sequence `seq` hold synthetic data;
    returns the arena and the stored row bytes [layer][token] for keys and values."""
    a = KvArena(ctx, model, layers, sequences, cap or tokens, kd, vd)
    hkv, d = a.hkv, a.d
    keys, vals = [], []
    for l in range(layers):
        kc = syn.normal(seed + 2 * l, (tokens, hkv, d))
        vc = syn.normal(seed + 2 * l + 1, (tokens, hkv, d))
        kc = kc if kd == F32 else (syn.to_bf16_bits(kc) if kd == BF16 else syn.to_f16_bits(kc))
        vc = vc if vd == F32 else (syn.to_bf16_bits(vc) if vd == BF16 else syn.to_f16_bits(vc))
        a.write(seq, l, 0, kc, vc)
        rk, rv = a.read(seq, l, 0, tokens)
        keys.append([rk[t].tobytes() for t in range(tokens)])
        vals.append([rv[t].tobytes() for t in range(tokens)])
    a.set_len(seq, tokens)
    return a, keys, vals


@pytest.mark.parametrize("layout", [HASH_PER_CHUNK, HASH_PER_SLOT])
@pytest.mark.parametrize("model,kd,vd", [(MODEL_GRANITE, F32, F32), (MODEL_GRANITE, BF16, BF16),
                                         (MODEL_GRANITE, F16, F16), (MODEL_GRANITE, F32, F16),
                                         (MODEL_GRANITE, F16, F32), (MODEL_QWEN3, BF16, BF16)])
def test_slot_hashes_match_oracle(gpu_ctx, oracle, model, kd, vd, layout):
    import torch
    layers, tokens = 3, 37  # ragged: 111 slots fill neither a warp nor a CTA evenly
    a, keys, vals = filled_arena(gpu_ctx, model, layers, tokens, kd, vd, 0x8100 + 16 * kd + vd)
    dig = torch.zeros(layers, tokens, 32, dtype=torch.uint8, device="cuda")
    a.slot_hashes(dig, 0, layers, 0, tokens, layout=layout)
    gpu_ctx.sync()
    got = dig.cpu().numpy()
    for l in range(layers):
        for t in range(tokens):
            assert got[l, t].tobytes() == oracle.kv_leaf_hash(l, t, keys[l][t], vals[l][t]), (l, t)


def test_slot_hashes_subrange_and_sequence(gpu_ctx, oracle):
    """A sub-range of layers and tokens of the second sequence: the leaves
    commit the absolute (layer, token) coordinates."""
    import torch
    layers, tokens = 4, 40
    a, keys, vals = filled_arena(gpu_ctx, MODEL_GRANITE, layers, tokens, BF16, BF16, 0x8200, seq=1, sequences=2,
                                 cap=64)
    for layout in (HASH_PER_CHUNK, HASH_PER_SLOT):
        dig = torch.zeros(2, 9, 32, dtype=torch.uint8, device="cuda")
        a.slot_hashes(dig, 1, 2, 30, 9, seq=1, layout=layout)
        gpu_ctx.sync()
        got = dig.cpu().numpy()
        for i in range(2):
            for j in range(9):
                l, t = 1 + i, 30 + j
                assert got[i, j].tobytes() == oracle.kv_leaf_hash(l, t, keys[l][t], vals[l][t])


def test_slot_hashes_full_context(gpu_ctx, oracle):
    """A whole 24-layer x 4096-token f32 Granite cache (98,304 slots, 402 MB
    hashed): every digest against the oracle."""
    import torch
    layers, tokens = 24, 4096
    a = KvArena(gpu_ctx, MODEL_GRANITE, layers, 1, tokens, F32, F32)
    gen = torch.Generator(device="cuda").manual_seed(0x8300)
    for l in range(layers):
        for key in (True, False):
            view = a.tensor(0, l, key).view(-1).view(torch.int32)
            view.copy_(torch.randint(-2**31, 2**31 - 1, view.shape, generator=gen, device="cuda",
                                     dtype=torch.int64).to(torch.int32))
    a.set_len(0, tokens)
    dig = torch.zeros(layers, tokens, 32, dtype=torch.uint8, device="cuda")
    a.slot_hashes(dig, 0, layers, 0, tokens)  # large enough for the lane-per-slot layout
    chunked = torch.zeros_like(dig)
    a.slot_hashes(chunked, 0, layers, 0, tokens, layout=HASH_PER_CHUNK)
    gpu_ctx.sync()
    assert torch.equal(dig, chunked)
    got = dig.cpu().numpy()
    assert len({got[l, t].tobytes() for l in range(layers) for t in range(tokens)}) == layers * tokens
    rng = np.random.default_rng(1)
    for l, t in [(0, 0), (23, 4095)] + [tuple(x) for x in rng.integers(0, [layers, tokens], (200, 2))]:
        k, v = a.read(0, int(l), int(t), 1)
        assert got[l, t].tobytes() == oracle.kv_leaf_hash(int(l), int(t), k.tobytes(), v.tobytes()), (l, t)


def test_verification_hashes_reference_golden_case(gpu_ctx, oracle):
    """qx-metal lib.rs:15531-15604 on the GPU: one f32 Granite layer, token
    11, checkpoint interval 1, snapshots 0 and 1 holding the same residual."""
    import torch
    residual = np.arange(1024, dtype=np.float32) * np.float32(0.125) - np.float32(64.0)
    key = np.arange(512, dtype=np.float32) * np.float32(-0.25) + np.float32(3.0)
    value = np.arange(512, dtype=np.float32) / np.float32(17.0)
    a = KvArena(gpu_ctx, MODEL_GRANITE, 1, 1, 16, F32, F32)
    a.write(0, 0, 11, key.reshape(1, 8, 64), value.reshape(1, 8, 64))
    a.set_len(0, 12)
    res = torch.from_numpy(np.concatenate([residual, residual])).cuda()
    dig = torch.zeros(2, 64, dtype=torch.uint8, device="cuda")
    a.verification_hashes(11, res, 4096, 1, dig)
    gpu_ctx.sync()
    got = dig.cpu().numpy().tobytes()
    want = oracle.verification_hashes(np.concatenate([residual, residual]).tobytes(), 4096, 1, 1,
                                      [key.tobytes()], [value.tobytes()], 11)
    assert got == want
    state = oracle.state_hash(residual.tobytes())
    assert got[:32] == state and got[32:64] == bytes(32) and got[64:96] == state
    assert got[96:] == oracle.kv_leaf_hash(0, 11, key.tobytes(), value.tobytes())


@pytest.mark.parametrize("kd,vd,stride,interval", [(F32, F32, 4096, 4), (BF16, BF16, 1024, 3),
                                                   (F32, F16, 256, 24), (F16, F16, 2048, 1)])
def test_verification_hashes_24_layers(gpu_ctx, oracle, kd, vd, stride, interval):
    """The reference's per-token call at its own shape (24 layers): state
    roots at checkpoint positions only, slot leaves of every layer."""
    import torch
    layers, tokens, token = 24, 20, 17
    a, keys, vals = filled_arena(gpu_ctx, MODEL_GRANITE, layers, tokens, kd, vd, 0x8400 + stride + interval)
    rng = np.random.default_rng(stride + interval)
    res = rng.integers(0, 256, (layers + 1) * stride, dtype=np.uint8)
    dig = torch.zeros(layers + 1, 64, dtype=torch.uint8, device="cuda")
    a.verification_hashes(token, torch.from_numpy(res).cuda(), stride, interval, dig)
    gpu_ctx.sync()
    want = oracle.verification_hashes(res.tobytes(), stride, interval, layers, [keys[l][token] for l in range(layers)],
                                      [vals[l][token] for l in range(layers)], token)
    assert dig.cpu().numpy().tobytes() == want


def test_verification_hashes_follow_decode(gpu_ctx, oracle):
    """A decode step then its commitments on the same stream: the hash reads
    the row the decode appended (the hash launch is a programmatic dependent
    of the decode)."""
    import torch
    prefix = 50
    kc, vc = syn.normal(0x8500, (prefix, 8, 64)), syn.normal(0x8501, (prefix, 8, 64))
    a = KvArena(gpu_ctx, MODEL_GRANITE, 1, 1, 64, F32, F32)
    a.write(0, 0, 0, kc, vc)
    a.set_len(0, prefix)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
    q, k, v = syn.normal(0x8502, (1024,)), syn.normal(0x8503, (512,)), syn.normal(0x8504, (512,))
    out = torch.zeros(1024, device="cuda")
    res = torch.from_numpy(syn.normal(0x8505, (2, 1024))).cuda()
    dig = torch.zeros(2, 64, dtype=torch.uint8, device="cuda")
    a.decode(dev(q), dev(k), dev(v), out, [prefix])
    a.verification_hashes(prefix, res, 4096, 1, dig)
    gpu_ctx.sync()
    rk, rv = a.read(0, 0, prefix, 1)
    want = oracle.verification_hashes(res.cpu().numpy().tobytes(), 4096, 1, 1, [rk.tobytes()], [rv.tobytes()], prefix)
    assert dig.cpu().numpy().tobytes() == want


def test_commitment_argument_errors(gpu_ctx):
    import torch
    a = KvArena(gpu_ctx, MODEL_GRANITE, 2, 1, 16, F32, F32)
    a.set_len(0, 4)
    res = torch.zeros(3, 1024, device="cuda")
    dig = torch.zeros(3, 64, dtype=torch.uint8, device="cuda")
    with pytest.raises(QxError, match="not below cache length 4"):
        a.verification_hashes(4, res, 4096, 1, dig)
    with pytest.raises(QxError, match="checkpoint interval 3 is outside 1..=2"):
        a.verification_hashes(0, res, 4096, 3, dig)
    with pytest.raises(QxError, match="residual size 768"):
        a.verification_hashes(0, res, 768, 1, dig)
    with pytest.raises(QxError, match="residual size 8192"):
        a.verification_hashes(0, res, 8192, 1, dig)
    with pytest.raises(QxError, match=r"tokens \[2, 6\) are not below cache length 4"):
        a.slot_hashes(dig, 0, 1, 2, 4)
    with pytest.raises(QxError, match="outside the arena's 2 layers"):
        a.slot_hashes(dig, 1, 2, 0, 1)
    with pytest.raises(QxError, match="unknown hash flags"):
        a.slot_hashes(dig, 0, 1, 0, 1, layout=3)
