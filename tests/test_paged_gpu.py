"""Paged KV arenas (qxc_kv_create_paged) against contiguous arenas.

A paged arena keeps per layer a pool of fixed-size pages shared by all
sequences and maps each sequence's logical pages through a block table. The
kernels compute exactly what they compute on a contiguous arena, only the row
addresses differ, so the gates are bit-identical outputs, rows and digests
(and, through the contiguous arena, the oracle parity of the other tests).
Pages are deliberately interleaved between sequences.
"""
import numpy as np
import pytest

from qx_b200 import BF16, F16, F32, MODEL_GRANITE, MODEL_QWEN3, KvArena, QxError
from qx_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def enc(x, dt):
    return x if dt == F32 else (syn.to_bf16_bits(x) if dt == BF16 else syn.to_f16_bits(x))


def twin_arenas(ctx, model, layers, lengths, kd, vd, page, pool, seed, capacity=None):
    """A contiguous and a paged arena holding the same rows; the paged one is
    filled page by page in round-robin over the sequences, so consecutive
    physical pages belong to different sequences."""
    cap = capacity or max(lengths) + 8
    a = KvArena(ctx, model, layers, len(lengths), cap, kd, vd)
    b = KvArena(ctx, model, layers, len(lengths), cap, kd, vd, page_size=page, pool_pages=pool)
    rows = {}
    for s, n in enumerate(lengths):
        for l in range(layers):
            kc = enc(syn.normal(seed + 100 * s + 2 * l, (n, a.hkv, a.d)), kd)
            vc = enc(syn.normal(seed + 100 * s + 2 * l + 1, (n, a.hkv, a.d)), vd)
            rows[s, l] = (kc, vc)
            if n:
                a.write(s, l, 0, kc, vc)
    for p in range((max(lengths) + page - 1) // page):
        for s, n in enumerate(lengths):
            lo, hi = p * page, min(n, (p + 1) * page)
            if lo < hi:
                for l in range(layers):
                    kc, vc = rows[s, l]
                    b.write(s, l, lo, kc[lo:hi], vc[lo:hi])
    for s, n in enumerate(lengths):
        a.set_len(s, n)
        b.set_len(s, n)
    return a, b


def same_rows(a, b, seqs, layers):
    for s in seqs:
        n = a.len(s)
        assert b.len(s) == n
        for l in range(layers):
            ak, av = a.read(s, l, 0, n)
            bk, bv = b.read(s, l, 0, n)
            assert np.array_equal(ak.view(np.uint8), bk.view(np.uint8)), (s, l)
            assert np.array_equal(av.view(np.uint8), bv.view(np.uint8)), (s, l)


@pytest.mark.parametrize("kd,vd,page", [(F32, F32, 64), (BF16, BF16, 64), (F16, F32, 128), (BF16, BF16, 256)])
def test_paged_granite_decode_matches_contiguous(gpu_ctx, kd, vd, page):
    """Ragged sequences, three decode steps; two sequences cross a page
    boundary on the way (63 -> 64 -> 65 and 127 -> 128 with 64-row pages)."""
    import torch
    lengths = [1, 63, 127, 200, 1000, 64]
    layers = 2
    a, b = twin_arenas(gpu_ctx, MODEL_GRANITE, layers, lengths, kd, vd, page, 64, 0x9100 + page + kd)
    n = len(lengths)
    for step in range(3):
        q = torch.from_numpy(syn.normal(0x9200 + step, (n, layers, 1024))).cuda()
        k = torch.from_numpy(syn.normal(0x9300 + step, (n, layers, 512))).cuda()
        v = torch.from_numpy(syn.normal(0x9400 + step, (n, layers, 512))).cuda()
        pos = [a.len(s) for s in range(n)]
        oa = torch.zeros(n, layers, 1024, device="cuda")
        ob = torch.zeros_like(oa)
        a.decode(q, k, v, oa, pos, split=64)
        b.decode(q, k, v, ob, pos, split=64)
        gpu_ctx.sync()
        assert torch.equal(oa, ob), step
    same_rows(a, b, range(n), layers)
    mapped = sum((a.len(s) + page - 1) // page for s in range(n))
    assert b.page_stats() == (mapped, 64 - mapped)


def test_paged_granite_decode_automatic_split_many_sequences(gpu_ctx):
    """A config-4-like batch: 48 sequences of lengths U{1..2048}, bf16 KV,
    4 layers in one call, the library's own split choice."""
    import torch
    rng = np.random.default_rng(7)
    lengths = [int(x) for x in rng.integers(1, 2049, 48)]
    layers = 4
    pool = sum((x + 1 + 63) // 64 for x in lengths) + 4
    a, b = twin_arenas(gpu_ctx, MODEL_GRANITE, layers, lengths, BF16, BF16, 64, pool, 0x9500, capacity=2100)
    n = len(lengths)
    q = torch.from_numpy(syn.normal(0x9600, (n, layers, 1024))).cuda()
    k = torch.from_numpy(syn.normal(0x9601, (n, layers, 512))).cuda()
    v = torch.from_numpy(syn.normal(0x9602, (n, layers, 512))).cuda()
    pos = [a.len(s) for s in range(n)]
    oa = torch.zeros(n, layers, 1024, device="cuda")
    ob = torch.zeros_like(oa)
    a.decode(q, k, v, oa, pos)
    split = gpu_ctx.last_split
    b.decode(q, k, v, ob, pos, split=split)
    gpu_ctx.sync()
    assert torch.equal(oa, ob)
    same_rows(a, b, [0, 17, 47], layers)


def test_paged_qwen_decode_matches_contiguous(gpu_ctx):
    import torch
    lengths = [130, 700, 5]
    a, b = twin_arenas(gpu_ctx, MODEL_QWEN3, 1, lengths, BF16, BF16, 64, 40, 0x9700)
    n = len(lengths)
    conv = lambda x: torch.from_numpy(syn.to_bf16_bits(x).view(np.int16)).cuda()
    qn = torch.from_numpy((1.0 + 0.1 * syn.normal(0x9710, (128,))).astype(np.float32)).cuda()
    kn = torch.from_numpy((1.0 + 0.1 * syn.normal(0x9711, (128,))).astype(np.float32)).cuda()
    for step in range(2):
        q = conv(syn.normal(0x9720 + step, (n, 1, 4096)))
        k = conv(syn.normal(0x9730 + step, (n, 1, 512)))
        v = conv(syn.normal(0x9740 + step, (n, 1, 512)))
        pos = [a.len(s) for s in range(n)]
        oa = torch.zeros(n, 1, 4096, device="cuda")
        ob = torch.zeros_like(oa)
        a.decode(q, k, v, oa, pos, q_norm=qn, k_norm=kn, split=128)
        b.decode(q, k, v, ob, pos, q_norm=qn, k_norm=kn, split=128)
        gpu_ctx.sync()
        assert torch.equal(oa, ob), step
    same_rows(a, b, range(n), 1)


def test_paged_verify_and_hashes_match_contiguous(gpu_ctx):
    """Four speculative tokens across a page boundary, then the slot
    commitments of every row of both sequences."""
    import torch
    lengths = [62, 300]
    a, b = twin_arenas(gpu_ctx, MODEL_GRANITE, 2, lengths, F32, F32, 64, 16, 0x9800)
    q = torch.from_numpy(syn.normal(0x9810, (4, 2, 1024))).cuda()
    k = torch.from_numpy(syn.normal(0x9811, (4, 2, 512))).cuda()
    v = torch.from_numpy(syn.normal(0x9812, (4, 2, 512))).cuda()
    oa = torch.zeros(4, 2, 1024, device="cuda")
    ob = torch.zeros_like(oa)
    a.decode_verify(q, k, v, oa, 62, 4, seq=0)
    b.decode_verify(q, k, v, ob, 62, 4, seq=0)
    gpu_ctx.sync()
    assert torch.equal(oa, ob)
    same_rows(a, b, [0, 1], 2)
    for s in (0, 1):
        n = a.len(s)
        da = torch.zeros(2, n, 32, dtype=torch.uint8, device="cuda")
        db = torch.zeros_like(da)
        a.slot_hashes(da, 0, 2, 0, n, seq=s)
        b.slot_hashes(db, 0, 2, 0, n, seq=s)
        gpu_ctx.sync()
        assert torch.equal(da, db)


def test_page_pool_exhaustion_reset_and_trim(gpu_ctx):
    import torch
    b = KvArena(gpu_ctx, MODEL_GRANITE, 1, 2, 512, F32, F32, page_size=64, pool_pages=4)
    b.set_len(0, 200)  # 4 pages: the whole pool
    assert b.page_stats(0) == (4, 0)
    z = torch.zeros(1, 1, 1024, device="cuda")
    zk = torch.zeros(1, 1, 512, device="cuda")
    launches = gpu_ctx.launch_count
    with pytest.raises(QxError, match="page pool exhausted"):
        b.decode(z, zk, zk, z, [0], seq_ids=[1])
    assert gpu_ctx.launch_count == launches and b.len(1) == 0
    # rollback keeps the pages for regrowth; trim returns the ones past the length
    b.rollback(0, 60)
    assert b.page_stats(0) == (4, 0)
    b.trim(0)
    assert b.page_stats(0) == (1, 3)
    b.decode(z, zk, zk, z, [0], seq_ids=[1])
    gpu_ctx.sync()
    assert b.len(1) == 1 and b.page_stats(1) == (1, 2)
    b.reset(0)
    assert b.page_stats(0) == (0, 3) and b.page_stats() == (1, 3)
    with pytest.raises(QxError, match="no contiguous view"):
        b.key_buffer(0, 0)
    with pytest.raises(QxError, match="not all mapped"):
        b.read(1, 0, 0, 65)


def test_paged_arena_rejects_bad_geometry(gpu_ctx):
    with pytest.raises(QxError, match="power of two"):
        KvArena(gpu_ctx, MODEL_GRANITE, 1, 1, 256, F32, F32, page_size=96, pool_pages=4)
    with pytest.raises(QxError, match="power of two"):
        KvArena(gpu_ctx, MODEL_GRANITE, 1, 1, 256, F32, F32, page_size=32, pool_pages=4)
    with pytest.raises(QxError, match="at least one page"):
        KvArena(gpu_ctx, MODEL_GRANITE, 1, 1, 256, F32, F32, page_size=64, pool_pages=0)
