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


@pytest.mark.parametrize("L", [1, 63, 64, 65, 200, 512])
def test_prefill_matches_iterated_decode(gpu_ctx, oracle, L):
    q, k, v, arena, got = run_prefill(gpu_ctx, L, syn.seed_for(2) + L)
    st, kc, vc, ref = oracle.granite_prefill(q, k, v, oracle.BF16, oracle.BF16, threads=8)
    assert st == 0
    assert normwise(got, ref) <= 2e-2
    gk, gv = arena.read(0, 0, 0, L)
    assert np.array_equal(gk, kc) and np.array_equal(gv, vc)
    assert arena.len(0) == L


@pytest.mark.slow
def test_prefill_2048(gpu_ctx, oracle):
    L = 2048
    q, k, v, arena, got = run_prefill(gpu_ctx, L, syn.seed_for(2))
    st, kc, vc, ref = oracle.granite_prefill(q, k, v, oracle.BF16, oracle.BF16, threads=8)
    assert st == 0
    assert normwise(got, ref) <= 2e-2
    gk, _ = arena.read(0, 0, 0, L)
    assert np.array_equal(gk, kc)


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
