"""One rank of a Qwen3 KV-length split, run under torchrun by
tests/test_exchange_gpu.py: each step decodes this rank's range and merges
the ranks' partials three ways, through qxc_exchange_merge (peer stores over
NVLink into CUDA IPC areas), through qxc_decode_exchange (the same exchange
inside the split merge kernel) and through the NCCL all-gather +
qxc_lse_merge; all three must agree bit for bit on every rank, and rank 0
checks them against one unsplit decode of the whole cache."""
import datetime
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main() -> int:
    import torch
    import torch.distributed as dist
    from qx_b200 import BF16, F32, MODEL_QWEN3, Context, KvArena
    from qx_b200 import synthetic as syn
    from qx_b200.distributed import all_gather_partials, kv_ranges, open_peer_group

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    ctx = Context(local)
    ctx.set_stream(torch.cuda.current_stream())
    # 128-row splits give every rank more than 8 splits up to 8 ranks, so
    # qxc_decode_partials and the fused exchange both combine them in the
    # split merge kernel (bit-identical paths)
    L0, steps, split = 12000, 3, 128
    L = L0 + steps
    b, e = kv_ranges(L, world)[rank]
    owner = rank == world - 1
    conv = syn.to_bf16_bits
    kc, vc = conv(syn.normal(0x6100, (L0, 4, 128))), conv(syn.normal(0x6101, (L0, 4, 128)))
    cached = min(e, L0) - b
    arenas = []
    for _ in range(2):  # one for the two-kernel paths, one for the fused exchange
        a = KvArena(ctx, MODEL_QWEN3, 1, 1, e - b, BF16, BF16, first_position=b)
        a.write(0, 0, 0, kc[b:b + cached], vc[b:b + cached])
        a.set_len(0, cached)
        arenas.append(a)
    arena, fused_arena = arenas
    group = open_peer_group(ctx)
    fused_group = open_peer_group(ctx)
    qs = [conv(syn.normal(0x6200 + t, (1, 4096))) for t in range(steps)]
    ks = [conv(syn.normal(0x6300 + t, (1, 512))) for t in range(steps)]
    vs = [conv(syn.normal(0x6400 + t, (1, 512))) for t in range(steps)]
    dv = lambda a: torch.from_numpy(a.view(np.int16)).to(dev)
    parts = torch.zeros(32, 130, device=dev)
    outs = []
    for t in range(steps):
        arena.decode_partials(dv(qs[t]), dv(ks[t]), dv(vs[t]), parts, L0 + t, append=owner, split=split)
        via_peers = torch.zeros(4096, device=dev)
        group.exchange_merge(MODEL_QWEN3, parts, via_peers)
        via_nccl = torch.zeros(4096, device=dev)
        ctx.lse_merge(MODEL_QWEN3, world, all_gather_partials(parts), via_nccl)
        ctx.sync()
        fused = torch.zeros(4096, device=dev)
        fused_arena.decode_exchange(dv(qs[t]), dv(ks[t]), dv(vs[t]), fused, L0 + t, append=owner, group=fused_group,
                                    split=split)
        ctx.sync()
        if not torch.equal(via_peers, via_nccl):
            print(f"rank {rank} step {t}: exchange differs from the NCCL path", flush=True)
            return 1
        if not torch.equal(fused, via_nccl):
            print(f"rank {rank} step {t}: fused exchange differs from the NCCL path", flush=True)
            return 1
        outs.append(via_peers.cpu().numpy())
    # every rank holds the same outputs
    gathered = [None] * world
    dist.all_gather_object(gathered, [o.tobytes() for o in outs])
    if any(g != gathered[0] for g in gathered):
        print(f"rank {rank}: ranks disagree", flush=True)
        return 1
    if rank == 0:
        whole = KvArena(ctx, MODEL_QWEN3, 1, 1, L, BF16, BF16)
        whole.write(0, 0, 0, kc, vc)
        whole.set_len(0, L0)
        for t in range(steps):
            ref = torch.zeros(1, 4096, device=dev)
            whole.decode(dv(qs[t]), dv(ks[t]), dv(vs[t]), ref, [L0 + t], out_dtype=F32)
            ctx.sync()
            r = ref.cpu().numpy()[0]
            err = float(np.max(np.abs(outs[t] - r)) / max(np.max(np.abs(r)), 1e-30))
            if err > 2e-2:  # the 16-bit KV gate: P is rounded to bf16 at other split points
                print(f"step {t}: split result off the unsplit decode by {err:.3g}", flush=True)
                return 1
        print(f"exchange ok: world {world}, {steps} steps", flush=True)
    dist.barrier()  # no rank closes its area while a peer may still store into it
    group.close()
    fused_group.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
