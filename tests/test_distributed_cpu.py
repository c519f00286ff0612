"""CPU tests of the multi-GPU host logic: LPT sharding, KV-length ranges, and
the partial exchange on world_size-2 gloo ranks, merged with the
log-sum-exp rule and checked against the unsplit oracle result."""
import os
import socket

import numpy as np
import pytest

from qx_b200 import synthetic as syn
from qx_b200.distributed import kv_ranges, lpt_shard, sequence_kv_bytes


def test_lpt_balances_config4_lengths():
    lengths = syn.uniform_int(0x51580400, 256, 128, 4096)
    costs = [sequence_kv_bytes(int(L)) for L in lengths]
    for n in (1, 2, 4, 8):
        assignment, loads = lpt_shard(costs, n)
        assert sorted(i for a in assignment for i in a) == list(range(256))
        assert max(loads) / (sum(costs) / n) < 1.01  # within 1% of perfect balance
        # deterministic
        assert lpt_shard(costs, n)[0] == assignment


def test_lpt_edge_cases():
    assert lpt_shard([], 3)[0] == [[], [], []]
    a, loads = lpt_shard([5, 5, 5], 2)
    assert sorted(loads) == [5, 10]
    with pytest.raises(ValueError):
        lpt_shard([1], 0)


def test_kv_ranges_cover_and_balance():
    for L, n in ((32768, 2), (32768, 8), (1000, 3), (7, 7)):
        r = kv_ranges(L, n)
        assert r[0][0] == 0 and r[-1][1] == L
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        assert max(e - b for b, e in r) - min(e - b for b, e in r) <= 1
    with pytest.raises(ValueError):
        kv_ranges(3, 4)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _shard_worker(rank, world, port, result_q):
    import sys
    import torch
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "oracle"))
    from qx_b200.distributed import all_gather_partials, kv_ranges
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    # each rank: partial (O, m, l) of Granite head attention over its KV range
    L = 300
    rng = np.random.default_rng(7)
    q = rng.standard_normal((16, 64)).astype(np.float32)
    k = rng.standard_normal((L, 8, 64)).astype(np.float32)
    v = rng.standard_normal((L, 8, 64)).astype(np.float32)
    b, e = kv_ranges(L, world)[rank]
    part = np.zeros((16, 66), np.float32)
    for h in range(16):
        s = (k[b:e, h // 2] @ q[h]) / 64.0
        m = s.max()
        w = np.exp(s - m)
        part[h, :64] = w @ v[b:e, h // 2]
        part[h, 64] = m
        part[h, 65] = w.sum()
    gathered = all_gather_partials(torch.from_numpy(part)).numpy()
    if rank == 0:
        M = gathered[:, :, 64].max(axis=0)
        scale = np.exp(gathered[:, :, 64] - M[None])
        out = (scale[:, :, None] * gathered[:, :, :64]).sum(0) / (scale * gathered[:, :, 65]).sum(0)[:, None]
        ref = np.zeros((16, 64), np.float32)
        for h in range(16):
            s = (k[:, h // 2] @ q[h]) / 64.0
            w = np.exp(s - s.max())
            ref[h] = (w @ v[:, h // 2]) / w.sum()
        result_q.put(float(np.abs(out - ref).max() / np.abs(ref).max()))
    dist.destroy_process_group()


def test_partial_exchange_two_gloo_ranks():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert q.get(timeout=5) < 1e-5


def _handle_worker(rank, world, port, result_q):
    """open_peer_group's host side: every rank's IPC handle reaches every
    other rank, which attaches it under the sender's rank (the CUDA calls are
    replaced by a recording stand-in)."""
    import sys
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import qx_b200.runtime as rt
    from qx_b200.distributed import open_peer_group
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)

    class Recorder:
        def __init__(self, ctx, r, w):
            self.rank, self.world, self.opened = r, w, {}

        def ipc_handle(self):
            return bytes([65 + self.rank]) * 64

        def open(self, peer, handle):
            self.opened[peer] = handle

    rt.PeerGroup = Recorder
    g = open_peer_group(None)
    result_q.put((rank, g.rank, g.world, sorted((p, h) for p, h in g.opened.items())))
    dist.destroy_process_group()


def test_peer_group_handles_three_gloo_ranks():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 3
    procs = [ctx.Process(target=_handle_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=5) for _ in range(world))
    for rank, grank, gworld, opened in got:
        assert (grank, gworld) == (rank, world)
        assert opened == [(p, bytes([65 + p]) * 64) for p in range(world) if p != rank]
