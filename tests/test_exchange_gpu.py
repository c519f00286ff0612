"""The NVLink exchange + merge of a KV-length split (qxc_exchange_merge)
against the all-gather + qxc_lse_merge path: bit-identical outputs.

One GPU covers a one-rank group (the phase alternation over steps) and the
bounded wait: a group of two whose second rank never runs must report
QXC_ERR_TIMEOUT at sync and leave the context usable. Two or more GPUs cover
the real exchange, in one process (qxc_peer_group_set_peer, peer access) and
as torchrun ranks (CUDA IPC), which is how the bench runs it.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from qx_b200 import BF16, F32, MODEL_GRANITE, MODEL_QWEN3, Context, KvArena, PeerGroup, QxError
from qx_b200 import synthetic as syn

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def qwen_shard(ctx, lo, hi, cached, seed, dev):
    conv = syn.to_bf16_bits
    kc, vc = conv(syn.normal(seed, (cached, 4, 128))), conv(syn.normal(seed + 1, (cached, 4, 128)))
    a = KvArena(ctx, MODEL_QWEN3, 1, 1, hi - lo, BF16, BF16, first_position=lo)
    a.write(0, 0, 0, kc, vc)
    a.set_len(0, cached)
    return a


def test_exchange_one_rank_equals_lse_merge(gpu_ctx):
    """world 1: the kernel's push, flag, wait and merge with itself, over
    five steps (both phases twice)."""
    import torch
    g = PeerGroup(gpu_ctx, 0, 1)
    a = qwen_shard(gpu_ctx, 0, 3000, 2990, 0x6500, "cuda")
    conv = lambda x: torch.from_numpy(syn.to_bf16_bits(x).view(np.int16)).cuda()
    parts = torch.zeros(32, 130, device="cuda")
    for t in range(5):
        q, k, v = conv(syn.normal(0x6510 + t, (1, 4096))), conv(syn.normal(0x6520 + t, (1, 512))), \
            conv(syn.normal(0x6530 + t, (1, 512)))
        a.decode_partials(q, k, v, parts, 2990 + t, append=True, split=256)
        x = torch.zeros(4096, device="cuda")
        y = torch.zeros(4096, device="cuda")
        g.exchange_merge(MODEL_QWEN3, parts, x)
        gpu_ctx.lse_merge(MODEL_QWEN3, 1, parts, y)
        gpu_ctx.sync()
        assert torch.equal(x, y), t
    g.close()


@pytest.mark.parametrize("model,rows,split", [(MODEL_QWEN3, 3000, 256), (MODEL_QWEN3, 100, 0),
                                              (MODEL_GRANITE, 1500, 128), (MODEL_GRANITE, 40, 0)])
def test_fused_exchange_one_rank_equals_partials_merge(gpu_ctx, model, rows, split):
    """qxc_decode_exchange with a one-rank group against qxc_decode_partials
    + qxc_lse_merge on a twin arena, over three steps; 100 and 40 rows are one
    split, which the fused path also sends through the split merge."""
    import torch
    qwen = model == MODEL_QWEN3
    hq, d, hkv = (32, 128, 4) if qwen else (16, 64, 8)
    dt = BF16 if qwen else F32
    enc = (lambda x: syn.to_bf16_bits(x)) if qwen else (lambda x: x)
    dv = (lambda x: torch.from_numpy(enc(x).view(np.int16)).cuda()) if qwen else (lambda x: torch.from_numpy(x).cuda())
    kc, vc = enc(syn.normal(0x6700, (rows, hkv, d))), enc(syn.normal(0x6701, (rows, hkv, d)))
    twins = []
    for _ in range(2):
        a = KvArena(gpu_ctx, model, 1, 1, rows + 8, dt, dt)
        a.write(0, 0, 0, kc, vc)
        a.set_len(0, rows)
        twins.append(a)
    g = PeerGroup(gpu_ctx, 0, 1)
    parts = torch.zeros(hq, d + 2, device="cuda")
    for t in range(3):
        q, k, v = syn.normal(0x6710 + t, (1, hq * d)), syn.normal(0x6720 + t, (1, hkv * d)), \
            syn.normal(0x6730 + t, (1, hkv * d))
        ref = torch.zeros(hq * d, device="cuda")
        twins[0].decode_partials(dv(q), dv(k), dv(v), parts, rows + t, append=True, split=split)
        gpu_ctx.lse_merge(model, 1, parts, ref)
        got = torch.zeros(hq * d, device="cuda")
        twins[1].decode_exchange(dv(q), dv(k), dv(v), got, rows + t, append=True, group=g, split=split)
        gpu_ctx.sync()
        assert torch.equal(got, ref), t
    ak, av = twins[0].read(0, 0, 0, rows + 3)
    bk, bv = twins[1].read(0, 0, 0, rows + 3)
    assert np.array_equal(ak, bk) and np.array_equal(av, bv)
    g.close()


def test_fused_exchange_missing_peer_times_out(gpu_ctx):
    import torch
    g0, g1 = PeerGroup(gpu_ctx, 0, 2), PeerGroup(gpu_ctx, 1, 2)
    g0.set_peer(1, g1.base())
    a = qwen_shard(gpu_ctx, 0, 2000, 1999, 0x6800, "cuda")
    conv = lambda x: torch.from_numpy(syn.to_bf16_bits(x).view(np.int16)).cuda()
    out = torch.zeros(4096, device="cuda")
    a.decode_exchange(conv(syn.normal(1, (1, 4096))), conv(syn.normal(2, (1, 512))), conv(syn.normal(3, (1, 512))),
                      out, 1999, append=True, group=g0, split=256)
    with pytest.raises(QxError, match="peer group is failed"):
        gpu_ctx.sync()
    # the heads' step counters no longer agree: the group refuses further use
    with pytest.raises(QxError, match="peer group failed"):
        a.decode_exchange(conv(syn.normal(4, (1, 4096))), conv(syn.normal(5, (1, 512))),
                          conv(syn.normal(6, (1, 512))), out, 2000, append=True, group=g0, split=256)
    g0.close()
    g1.close()


def test_exchange_missing_peer_times_out(gpu_ctx):
    """Rank 0 of two, the second rank's area attached but never run: every
    head's wait runs out (about a second), sync reports the timeout, the peer
    group is failed from then on (an exchange already enqueued does nothing,
    a later call is refused), and the context keeps working."""
    import torch
    g0, g1 = PeerGroup(gpu_ctx, 0, 2), PeerGroup(gpu_ctx, 1, 2)
    g0.set_peer(1, g1.base())
    parts = torch.zeros(32, 130, device="cuda")
    parts[:, 128] = 0.0   # m
    parts[:, 129] = 1.0   # l
    out = torch.zeros(4096, device="cuda")
    g0.exchange_merge(MODEL_QWEN3, parts, out)
    # enqueued before the failure is known: its kernel finds the group failed
    # and returns at once, pushing and merging nothing
    out2 = torch.full((4096,), 7.0, device="cuda")
    g0.exchange_merge(MODEL_QWEN3, parts, out2)
    with pytest.raises(QxError, match="peer group is failed"):
        gpu_ctx.sync()
    assert torch.all(out2 == 7.0)
    # after the failure is recorded, the group refuses every exchange call
    with pytest.raises(QxError, match="peer group failed"):
        g0.exchange_merge(MODEL_QWEN3, parts, out)
    y = torch.zeros(4096, device="cuda")
    gpu_ctx.lse_merge(MODEL_QWEN3, 1, parts, y)
    gpu_ctx.sync()
    assert torch.equal(y, torch.zeros_like(y))
    g0.close()
    g1.close()


def test_exchange_rejects_unattached_peer(gpu_ctx):
    import torch
    g = PeerGroup(gpu_ctx, 0, 2)
    with pytest.raises(QxError, match="peer 1 is not attached"):
        g.exchange_merge(MODEL_QWEN3, torch.zeros(32, 130, device="cuda"), torch.zeros(4096, device="cuda"))
    with pytest.raises(QxError, match="not another rank"):
        g.set_peer(0, g.base())
    g.close()


def test_exchange_two_gpus_one_process():
    """Ranks 0 and 1 on GPUs 0 and 1, driven from one process: each rank's
    kernel runs on its own GPU, so the two that wait on each other run at
    the same time. 128-row splits give each shard 16 splits, so the split
    partials of both paths are combined by the split merge kernel."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctxs = [Context(i) for i in range(2)]
    streams = [torch.cuda.Stream(device=i) for i in range(2)]
    for c, s in zip(ctxs, streams):
        c.set_stream(s)
    groups = [PeerGroup(ctxs[i], i, 2) for i in range(2)]
    groups[0].set_peer(1, groups[1].base())
    groups[1].set_peer(0, groups[0].base())
    L = 4000
    arenas = [qwen_shard(ctxs[0], 0, 2000, 2000, 0x6600, "cuda:0"),
              qwen_shard(ctxs[1], 2000, 4001, 1999, 0x6602, "cuda:1")]
    conv = syn.to_bf16_bits
    q, k, v = conv(syn.normal(0x6610, (1, 4096))), conv(syn.normal(0x6611, (1, 512))), conv(syn.normal(0x6612, (1, 512)))
    outs, parts = [], []
    for i in range(2):
        dev = f"cuda:{i}"
        dv = lambda a: torch.from_numpy(a.view(np.int16)).to(dev)
        with torch.cuda.device(i), torch.cuda.stream(streams[i]):
            p = torch.zeros(32, 130, device=dev)
            arenas[i].decode_partials(dv(q), dv(k), dv(v), p, L - 1, append=(i == 1), split=128)
            parts.append(p)
            outs.append(torch.zeros(4096, device=dev))
    for i in range(2):
        groups[i].exchange_merge(MODEL_QWEN3, parts[i], outs[i])
    for c in ctxs:
        c.sync()
    with torch.cuda.device(0):
        both = torch.stack([parts[0], parts[1].to("cuda:0")])
        ref = torch.zeros(4096, device="cuda:0")
        ctxs[0].lse_merge(MODEL_QWEN3, 2, both, ref)
        ctxs[0].sync()
    assert torch.equal(outs[0], ref)
    assert torch.equal(outs[1].to("cuda:0"), ref)
    # the same step fused into the split merge, on twin shards
    fgroups = [PeerGroup(ctxs[i], i, 2) for i in range(2)]
    fgroups[0].set_peer(1, fgroups[1].base())
    fgroups[1].set_peer(0, fgroups[0].base())
    twins = [qwen_shard(ctxs[0], 0, 2000, 2000, 0x6600, "cuda:0"),
             qwen_shard(ctxs[1], 2000, 4001, 1999, 0x6602, "cuda:1")]
    fouts = []
    for i in range(2):
        dev = f"cuda:{i}"
        dv = lambda a: torch.from_numpy(a.view(np.int16)).to(dev)
        with torch.cuda.device(i), torch.cuda.stream(streams[i]):
            fouts.append(torch.zeros(4096, device=dev))
            twins[i].decode_exchange(dv(q), dv(k), dv(v), fouts[i], L - 1, append=(i == 1), group=fgroups[i],
                                     split=128)
    for c in ctxs:
        c.sync()
    assert torch.equal(fouts[0], ref)
    assert torch.equal(fouts[1].to("cuda:0"), ref)
    for g in groups + fgroups:
        g.close()
    for c in ctxs:
        c.close()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_exchange_torchrun_ranks(world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={29640 + world}",
           os.path.join(ROOT, "tests", "exchange_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert f"exchange ok: world {world}" in r.stdout
