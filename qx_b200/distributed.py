"""Multi-GPU host logic for the attention path (one process per GPU).

Two ways the path spreads over GPUs of one node:

* Independent sequences (BASELINE configs 1 and 4): sequences are assigned
  to ranks by LPT (longest processing time first) on their KV bytes; each
  rank decodes its own sequences with no collective on the data path.
* One long context (config 3): the KV length is split into contiguous
  position ranges, one per rank; the last range owns the new token (RoPE +
  append). Each rank computes per-query-head partials (O, m, l) over its
  range with qxc_decode_partials; the partials ([q_heads][head_dim + 2]
  f32, 16,640 bytes per rank for Qwen3) are exchanged over NVLink and
  merged: qxc_exchange_merge pushes them into every rank's memory with peer
  stores and merges in one kernel (open_peer_group sets it up); the NCCL
  all-gather + qxc_lse_merge path (all_gather_partials) gives the same bits.
"""
from __future__ import annotations

import heapq


def lpt_shard(costs, n_ranks: int):
    """Assign items to ranks, largest cost first onto the least-loaded rank.

    Returns (assignment, loads): assignment[r] is the sorted list of item
    indices of rank r. Ties go to the lower rank, so the result is
    deterministic on every rank."""
    if n_ranks < 1:
        raise ValueError("n_ranks must be >= 1")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0, r) for r in range(n_ranks)]
    assignment = [[] for _ in range(n_ranks)]
    for i in order:
        load, r = heapq.heappop(heap)
        assignment[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    loads = [0] * n_ranks
    for r, items in enumerate(assignment):
        items.sort()
        loads[r] = sum(costs[i] for i in items)
    return assignment, loads


def sequence_kv_bytes(length: int, layers: int = 24, kv_heads: int = 8, head_dim: int = 64,
                      elem_bytes: int = 2) -> int:
    """KV bytes one decode step reads for a sequence of `length` positions."""
    return layers * 2 * length * kv_heads * head_dim * elem_bytes


def kv_ranges(length: int, n_ranks: int):
    """Contiguous, balanced [begin, end) position ranges covering 0..length-1."""
    if length < n_ranks:
        raise ValueError("need at least one position per rank")
    return [(length * r // n_ranks, length * (r + 1) // n_ranks) for r in range(n_ranks)]


def all_gather_partials(partials, group=None):
    """All-gather one rank's partial tensor (any shape) into [world, *shape]."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    flat = partials.contiguous().reshape(-1)
    out = torch.empty((world * flat.numel(),), dtype=partials.dtype, device=partials.device)
    dist.all_gather_into_tensor(out, flat, group=group)  # rank-major concatenation
    return out.view(world, *partials.shape)


def exchange_handles(local: bytes, group=None) -> list:
    """Every rank's bytes, in rank order (all_gather_object on the process group)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, local, group=group)
    return out


def open_peer_group(ctx, group=None):
    """Create this rank's qx_b200.PeerGroup and attach every other rank's area
    through CUDA IPC handles exchanged over the process group."""
    import torch.distributed as dist
    from .runtime import PeerGroup
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    pg = PeerGroup(ctx, rank, world)
    handles = exchange_handles(pg.ipc_handle(), group)
    for r, h in enumerate(handles):
        if r != rank:
            pg.open(r, h)
    dist.barrier(group)
    return pg
