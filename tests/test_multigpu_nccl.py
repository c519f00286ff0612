"""Two-rank NCCL test of the KV-length split (BASELINE config 3 shape, reduced
length): each rank holds a contiguous slice of one Qwen3 sequence's cache,
computes (O, m, l) partials with qxc_decode_partials, the partials are
all-gathered over NCCL and merged with qxc_lse_merge; rank 0 compares with
the single-arena decode. Skipped when fewer than two GPUs are visible."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_q):
    import sys
    import datetime
    import torch
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    from qx_b200 import BF16, MODEL_QWEN3, Context, KvArena
    from qx_b200 import synthetic as syn
    from qx_b200.distributed import all_gather_partials, kv_ranges
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        L = 5000
        P = L - 1
        conv = syn.to_bf16_bits
        q = conv(syn.normal(11, (32, 128)))
        k = conv(syn.normal(12, (4, 128)))
        v = conv(syn.normal(13, (4, 128)))
        kc = conv(syn.normal(14, (P, 4, 128)))
        vc = conv(syn.normal(15, (P, 4, 128)))
        dev = lambda a: torch.from_numpy(a.view(np.int16).reshape(1, -1)).cuda()
        ctx = Context(rank)
        ctx.set_stream(torch.cuda.current_stream())
        b, e = kv_ranges(L, world)[rank]
        cached = min(e, P) - b
        arena = KvArena(ctx, MODEL_QWEN3, 1, 1, e - b, BF16, BF16, first_position=b)
        arena.write(0, 0, 0, kc[b:b + cached], vc[b:b + cached])
        arena.set_len(0, cached)
        parts = torch.zeros(32, 130, device="cuda")
        arena.decode_partials(dev(q), dev(k), dev(v), parts, P, append=(rank == world - 1))
        allp = all_gather_partials(parts)
        merged = torch.zeros(4096, device="cuda")
        ctx.lse_merge(MODEL_QWEN3, world, allp, merged)
        ctx.sync()
        if rank == 0:
            whole = KvArena(ctx, MODEL_QWEN3, 1, 1, L, BF16, BF16)
            whole.write(0, 0, 0, kc, vc)
            whole.set_len(0, P)
            ref = torch.zeros(1, 4096, device="cuda")
            whole.decode(dev(q), dev(k), dev(v), ref, [P])
            ctx.sync()
            m, r = merged.cpu().numpy(), ref.cpu().numpy()[0]
            result_q.put(float(np.abs(m - r).max() / np.abs(r).max()))
        arena.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


def test_kv_split_two_gpus_nccl_merge():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import multiprocessing as mp
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _free_port()
    procs = [mpc.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    assert q.get(timeout=10) <= 2e-3
