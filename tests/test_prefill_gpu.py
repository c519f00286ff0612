"""GPU parity of the causal prefill against the oracle,
which defines prefill as granite_attention_decode iterated over positions
0..L-1 (the reference prefills a prompt token by token)."""
import numpy as np
import pytest

from helpers import normwise
from qx_b200 import BF16, F32, MODEL_GRANITE, KvArena, QxError
from qx_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def run_prefill(ctx, L, seed):
    import torch
    q = syn.to_bf16_bits(syn.normal(seed, (L, 16, 64), 0.5))
    k = syn.to_bf16_bits(syn.normal(seed + 1, (L, 8, 64), 0.5))
    v = syn.to_bf16_bits(syn.normal(seed + 2, (L, 8, 64), 0.5))
    arena = KvArena(ctx, MODEL_GRANITE, 1, 1, L + 64, BF16, BF16)
    dev = lambda a: torch.from_numpy(a.view(np.int16)).cuda()
    out = torch.zeros(L, 16, 64, device="cuda")
    arena.prefill(dev(q), dev(k), dev(v), out, L)
    ctx.sync()
    return q, k, v, arena, out.cpu().numpy()


@pytest.mark.parametrize("L", [1, 63, 64, 65, 128, 129, 200, 512, 1000])
def test_prefill_matches_iterated_decode(gpu_ctx, oracle, L):
    q, k, v, arena, got = run_prefill(gpu_ctx, L, syn.seed_for(2) + L)
    st, kc, vc, ref = oracle.granite_prefill(q, k, v, oracle.BF16, oracle.BF16, threads=8)
    assert st == 0
    assert normwise(got, ref) <= 2e-2
    gk, gv = arena.read(0, 0, 0, L)
    assert np.array_equal(gk, kc) and np.array_equal(gv, vc)
    assert arena.len(0) == L


@pytest.mark.parametrize("L", [1153, 1800, 2047, 2300])
def test_prefill_paired_blocks(gpu_ctx, oracle, L):
    """Lengths around the paired grid on 148 SMs. 1153 (19 blocks): a second
    wave of 4 CTAs, left unpaired. 1800 (29 blocks): paired, CTA j runs query
    blocks 28-j and j of one kv head back to back, the middle block alone.
    2047: paired, with a ragged last block. 2300 (36 blocks): the largest
    paired grid."""
    q, k, v, arena, got = run_prefill(gpu_ctx, L, syn.seed_for(2) + 7 * L)
    st, kc, vc, ref = oracle.granite_prefill(q, k, v, oracle.BF16, oracle.BF16, threads=8)
    assert st == 0
    assert normwise(got, ref) <= 2e-2
    gk, gv = arena.read(0, 0, 0, L)
    assert np.array_equal(gk, kc) and np.array_equal(gv, vc)


@pytest.mark.parametrize("L", [200, 2047])
def test_prefill_bf16_output(gpu_ctx, oracle, L):
    """The bf16 output rows (unpaired and paired grids) against the oracle."""
    import torch
    q = syn.to_bf16_bits(syn.normal(0x5200 + L, (L, 16, 64), 0.5))
    k = syn.to_bf16_bits(syn.normal(0x5201 + L, (L, 8, 64), 0.5))
    v = syn.to_bf16_bits(syn.normal(0x5202 + L, (L, 8, 64), 0.5))
    arena = KvArena(gpu_ctx, MODEL_GRANITE, 1, 1, L, BF16, BF16)
    dev = lambda a: torch.from_numpy(a.view(np.int16)).cuda()
    out = torch.zeros(L, 16, 64, device="cuda", dtype=torch.bfloat16)
    arena.prefill(dev(q), dev(k), dev(v), out, L, out_dtype=BF16)
    gpu_ctx.sync()
    st, _, _, ref = oracle.granite_prefill(q, k, v, oracle.BF16, oracle.BF16, threads=8)
    assert st == 0
    assert normwise(out.float().cpu().numpy(), ref) <= 2e-2


@pytest.mark.slow
def test_prefill_2048(gpu_ctx, oracle):
    L = 2048
    q, k, v, arena, got = run_prefill(gpu_ctx, L, syn.seed_for(2))
    st, kc, vc, ref = oracle.granite_prefill(q, k, v, oracle.BF16, oracle.BF16, threads=8)
    assert st == 0
    assert normwise(got, ref) <= 2e-2
    gk, _ = arena.read(0, 0, 0, L)
    assert np.array_equal(gk, kc)


def test_prefills_back_to_back(gpu_ctx, oracle):
    """Three prompts queued with no host sync between them, into three
    sequences of one arena (the RoPE grid of each may start its attention
    grid early, and reuses the context's rotated-query scratch): each must
    match the oracle."""
    import torch
    lengths = [700, 300, 700]
    arena = KvArena(gpu_ctx, MODEL_GRANITE, 1, 3, 768, BF16, BF16)
    dev = lambda a: torch.from_numpy(a.view(np.int16)).cuda()
    cases = []
    for s_, L in enumerate(lengths):
        q = syn.to_bf16_bits(syn.normal(0x5100 + s_, (L, 16, 64), 0.5))
        k = syn.to_bf16_bits(syn.normal(0x5200 + s_, (L, 8, 64), 0.5))
        v = syn.to_bf16_bits(syn.normal(0x5300 + s_, (L, 8, 64), 0.5))
        out = torch.zeros(L, 16, 64, device="cuda")
        arena.prefill(dev(q), dev(k), dev(v), out, L, seq=s_)
        cases.append((q, k, v, out))
    gpu_ctx.sync()
    for s_, (q, k, v, out) in enumerate(cases):
        st, kc, vc, ref = oracle.granite_prefill(q, k, v, oracle.BF16, oracle.BF16, threads=8)
        assert st == 0
        assert normwise(out.cpu().numpy(), ref) <= 2e-2, s_
        gk, gv = arena.read(s_, 0, 0, lengths[s_])
        assert np.array_equal(gk, kc) and np.array_equal(gv, vc)


def test_decode_continues_after_prefill(gpu_ctx, oracle):
    L = 100
    q, k, v, arena, _ = run_prefill(gpu_ctx, L, 0x777)
    st, kc, vc, _ = oracle.granite_prefill(q, k, v, oracle.BF16, oracle.BF16, threads=4)
    oc = oracle.KvCache(128, oracle.BF16, oracle.BF16)
    oc.keys[:L], oc.values[:L] = kc, vc
    oc.length.value = L
    qn, kn, vn = syn.normal(1, (1024,)), syn.normal(2, (512,)), syn.normal(3, (512,))
    st, ref = oracle.granite_attention_decode(qn, kn, vn, L, oc)
    out = arena.decode_host(qn[None], kn[None], vn[None], [L])[0]
    assert normwise(out, ref) <= 2e-2


def test_prefill_requires_empty_cache(gpu_ctx):
    import torch
    arena = KvArena(gpu_ctx, MODEL_GRANITE, 1, 1, 64, BF16, BF16)
    arena.set_len(0, 3)
    z = torch.zeros(8, 16, 64, dtype=torch.int16, device="cuda")
    with pytest.raises(QxError):
        arena.prefill(z, z[:, :8], z[:, :8], torch.zeros(8, 16, 64, device="cuda"), 8)
