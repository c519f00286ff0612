"""Speculative K-wide verify (qxc_decode_verify) against K successive decodes
and against the oracle iterated token by token.

The reference verifies K candidates in one pass (qx-runtime-v2
lib.rs:3722-3760: batched RoPE/KV append, then token t attends positions
[0, start + t]); the cursor keeps the accepted prefix through
checkpoint / commit (lib.rs:3265-3310). Gates as for decode: cache rows
bit-exact, outputs within 1e-5 (fp32 KV) / 2e-2 (16-bit KV) normwise.
"""
import numpy as np
import pytest

from helpers import as_kv, normwise
from qx_b200 import BF16, F16, F32, MODEL_GRANITE, MODEL_QWEN3, KvArena, QxError
from qx_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def granite_case(seed, prefix, tokens, layers):
    kc = syn.normal(seed, (layers, prefix, 8, 64))
    vc = syn.normal(seed + 1, (layers, prefix, 8, 64))
    q = syn.normal(seed + 2, (tokens, layers, 1024))
    k = syn.normal(seed + 3, (tokens, layers, 512))
    v = syn.normal(seed + 4, (tokens, layers, 512))
    return kc, vc, q, k, v


def filled(ctx, model, layers, cap, kd, vd, kc, vc):
    a = KvArena(ctx, model, layers, 1, cap, kd, vd)
    for l in range(layers):
        a.write(0, l, 0, kc[l], vc[l])
    a.set_len(0, kc.shape[1])
    return a


@pytest.mark.parametrize("prefix,tokens", [(0, 1), (0, 4), (37, 4), (63, 2), (500, 4), (1023, 3)])
def test_granite_verify_equals_successive_decodes(gpu_ctx, oracle, prefix, tokens):
    import torch
    layers, cap = 2, 1100
    kc, vc, q, k, v = granite_case(0x7100 + prefix, prefix, tokens, layers)
    a = filled(gpu_ctx, MODEL_GRANITE, layers, cap, F32, F32, kc, vc)
    b = filled(gpu_ctx, MODEL_GRANITE, layers, cap, F32, F32, kc, vc)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
    out = torch.zeros(tokens, layers, 1024, device="cuda")
    a.decode_verify(dev(q), dev(k), dev(v), out, prefix, tokens)
    seq = torch.zeros(tokens, layers, 1024, device="cuda")
    for t in range(tokens):
        b.decode(dev(q[t]), dev(k[t]), dev(v[t]), seq[t], [prefix + t])
    gpu_ctx.sync()
    assert a.len(0) == prefix + tokens == b.len(0)
    for l in range(layers):
        ak, av = a.read(0, l, 0, prefix + tokens)
        bk, bv = b.read(0, l, 0, prefix + tokens)
        assert np.array_equal(ak.view(np.uint32), bk.view(np.uint32))
        assert np.array_equal(av.view(np.uint32), bv.view(np.uint32))
    got = out.cpu().numpy()
    assert normwise(got, seq.cpu().numpy()) <= 1e-5
    # the oracle, token by token, per layer
    for l in range(layers):
        c = oracle.KvCache(cap)
        c.keys[:prefix], c.values[:prefix] = kc[l], vc[l]
        c.length.value = prefix
        for t in range(tokens):
            st, ref = oracle.granite_attention_decode(q[t, l], k[t, l], v[t, l], prefix + t, c)
            assert st == 0
            assert normwise(got[t, l], ref) <= 1e-5
        ak, _ = a.read(0, l, 0, prefix + tokens)
        assert np.array_equal(ak.view(np.uint32), c.keys[:prefix + tokens].view(np.uint32))


def test_granite_verify_bf16_kv(gpu_ctx):
    import torch
    prefix, tokens, cap = 300, 4, 320
    kc, vc, q, k, v = granite_case(0x7200, prefix, tokens, 1)
    a = filled(gpu_ctx, MODEL_GRANITE, 1, cap, BF16, BF16, as_kv(kc, BF16), as_kv(vc, BF16))
    b = filled(gpu_ctx, MODEL_GRANITE, 1, cap, BF16, BF16, as_kv(kc, BF16), as_kv(vc, BF16))
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
    out = torch.zeros(tokens, 1, 1024, device="cuda")
    a.decode_verify(dev(q), dev(k), dev(v), out, prefix, tokens)
    seq = torch.zeros(tokens, 1, 1024, device="cuda")
    for t in range(tokens):
        b.decode(dev(q[t]), dev(k[t]), dev(v[t]), seq[t], [prefix + t])
    gpu_ctx.sync()
    ak, av = a.read(0, 0, 0, prefix + tokens)
    bk, bv = b.read(0, 0, 0, prefix + tokens)
    assert np.array_equal(ak, bk) and np.array_equal(av, bv)
    assert normwise(out.cpu().numpy(), seq.cpu().numpy()) <= 2e-2


def test_qwen_verify_equals_successive_decodes(gpu_ctx):
    import torch
    prefix, tokens, cap = 700, 3, 720
    conv = syn.to_bf16_bits
    kc = conv(syn.normal(0x7300, (1, prefix, 4, 128)))
    vc = conv(syn.normal(0x7301, (1, prefix, 4, 128)))
    q = conv(syn.normal(0x7302, (tokens, 1, 4096)))
    k = conv(syn.normal(0x7303, (tokens, 1, 512)))
    v = conv(syn.normal(0x7304, (tokens, 1, 512)))
    qn = torch.from_numpy((1.0 + 0.1 * syn.normal(0x7305, (128,))).astype(np.float32)).cuda()
    kn = torch.from_numpy((1.0 + 0.1 * syn.normal(0x7306, (128,))).astype(np.float32)).cuda()
    a = filled(gpu_ctx, MODEL_QWEN3, 1, cap, BF16, BF16, kc, vc)
    b = filled(gpu_ctx, MODEL_QWEN3, 1, cap, BF16, BF16, kc, vc)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda()
    out = torch.zeros(tokens, 1, 4096, device="cuda")
    a.decode_verify(dev(q), dev(k), dev(v), out, prefix, tokens, q_norm=qn, k_norm=kn, split=128)
    seq = torch.zeros(tokens, 1, 4096, device="cuda")
    for t in range(tokens):
        b.decode(dev(q[t]), dev(k[t]), dev(v[t]), seq[t], [prefix + t], q_norm=qn, k_norm=kn, split=128)
    gpu_ctx.sync()
    ak, av = a.read(0, 0, 0, prefix + tokens)
    bk, bv = b.read(0, 0, 0, prefix + tokens)
    assert np.array_equal(ak, bk), "appended keys must be bit-identical to the decode's"
    assert np.array_equal(av, bv)
    assert normwise(out.cpu().numpy(), seq.cpu().numpy()) <= 2e-3


def test_verify_then_commit_accepted_prefix(gpu_ctx, oracle):
    """checkpoint -> verify 4 candidates -> commit 2: the cursor keeps the
    accepted prefix and the next decode continues from it."""
    import torch
    prefix, tokens, cap = 200, 4, 256
    kc, vc, q, k, v = granite_case(0x7400, prefix, tokens, 1)
    a = filled(gpu_ctx, MODEL_GRANITE, 1, cap, F32, F32, kc, vc)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
    cp = a.checkpoint(0)
    out = torch.zeros(tokens, 1, 1024, device="cuda")
    a.decode_verify(dev(q), dev(k), dev(v), out, prefix, tokens)
    gpu_ctx.sync()
    assert a.len(0) == prefix + tokens
    a.commit(0, cp, 2)
    assert a.len(0) == prefix + 2
    # the next token lands at prefix + 2 and sees the two accepted rows only
    q2, k2, v2 = syn.normal(0x7410, (1024,)), syn.normal(0x7411, (512,)), syn.normal(0x7412, (512,))
    got = a.decode_host(q2[None], k2[None], v2[None], [prefix + 2])[0]
    c = oracle.KvCache(cap)
    c.keys[:prefix], c.values[:prefix] = kc[0], vc[0]
    c.length.value = prefix
    for t in range(2):
        assert oracle.granite_attention_decode(q[t, 0], k[t, 0], v[t, 0], prefix + t, c)[0] == 0
    st, ref = oracle.granite_attention_decode(q2, k2, v2, prefix + 2, c)
    assert st == 0
    assert normwise(got, ref) <= 1e-5


def test_verify_rejects_bad_positions(gpu_ctx):
    import torch
    a = KvArena(gpu_ctx, MODEL_GRANITE, 1, 1, 8, F32, F32)
    a.set_len(0, 5)
    z = torch.zeros(4, 1, 1024, device="cuda")
    zk = torch.zeros(4, 1, 512, device="cuda")
    with pytest.raises(QxError, match="does not follow cache length 5"):
        a.decode_verify(z, zk, zk, z, 4, 2)
    with pytest.raises(QxError, match="exceeds context 8"):
        a.decode_verify(z, zk, zk, z, 5, 4)
    with pytest.raises(QxError, match="at least one token"):
        a.decode_verify(z, zk, zk, z, 5, 0)
    assert a.len(0) == 5


@pytest.mark.parametrize("prefix,tokens,split", [(300, 4, 64), (4000, 4, 0), (4000, 3, 64), (126, 2, 64),
                                                 (2000, 4, 2048)])
@pytest.mark.parametrize("kd,vd", [(F32, F32), (BF16, BF16), (F16, F32)])
def test_shared_tile_verify_equals_per_token(gpu_ctx, prefix, tokens, split, kd, vd):
    """2..4 Granite candidates share every cache tile (one work item per
    layer, kv head and split); against one causal decode entry per
    candidate (QXC_VERIFY_PER_TOKEN): rows bit-identical, outputs within
    fp32 rounding. Splits cover the in-kernel merge (5 splits), the
    separate merge (63) and one split; the draft crosses a 64-row tile."""
    import torch
    from helpers import as_kv
    from qx_b200._lib import VERIFY_PER_TOKEN
    layers, cap = 2, 4096
    kc, vc, q, k, v = granite_case(0x7500 + prefix + tokens, prefix, tokens, layers)
    kc, vc = as_kv(kc, kd), as_kv(vc, vd)
    a = filled(gpu_ctx, MODEL_GRANITE, layers, cap, kd, vd, kc, vc)
    b = filled(gpu_ctx, MODEL_GRANITE, layers, cap, kd, vd, kc, vc)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
    oa = torch.zeros(tokens, layers, 1024, device="cuda")
    ob = torch.zeros_like(oa)
    a.decode_verify(dev(q), dev(k), dev(v), oa, prefix, tokens, split=split)
    b.decode_verify(dev(q), dev(k), dev(v), ob, prefix, tokens, split=split, flags=VERIFY_PER_TOKEN)
    gpu_ctx.sync()
    for l in range(layers):
        ak, av = a.read(0, l, 0, prefix + tokens)
        bk, bv = b.read(0, l, 0, prefix + tokens)
        assert np.array_equal(ak, bk) and np.array_equal(av, bv)
    tol = 1e-5 if kd == F32 and vd == F32 else 2e-2
    assert normwise(oa.cpu().numpy(), ob.cpu().numpy()) <= tol
    assert torch.isfinite(oa).all()
