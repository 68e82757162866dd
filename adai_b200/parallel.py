"""Batch sharding across GPUs for the decode path: one process per GPU, each sequence on exactly
one rank, no collective on the data path.

Each sequence's decode depends only on its own tokens, encoder output and KV cache; the weights
are read-only. So a batch splits into per-rank shards. Rank r owns a contiguous range of the
global batch (sequence b goes to rank floor(b * world / B)). Optionally, shards are balanced by
source length, because the cross-attention bytes per step grow with it. Every rank decodes its
shard on its own device. The host then gathers the token ids (a few bytes per sequence per step)
to rank 0, which puts them back in batch order. Timing uses the maximum over ranks.

The process-group calls used here (all_gather_object, all_reduce) run on the host's gloo or
nccl group and move only ids and timings.
"""
from __future__ import annotations

from typing import Callable, Sequence


def shard_ranges(n: int, world: int) -> list[tuple[int, int]]:
    """Contiguous [lo, hi) per rank. Item b goes to rank floor(b * world / n), so shard sizes
    differ by at most one."""
    if world < 1 or n < 0:
        raise ValueError("need world >= 1 and n >= 0")
    owner = [b * world // n for b in range(n)] if n else []
    out = []
    for r in range(world):
        idx = [b for b in range(n) if owner[b] == r]
        out.append((idx[0], idx[-1] + 1) if idx else (n, n))
    return out


def balanced_shards(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Assigns items to ranks so that the per-rank sums of `lengths` (source lengths: the
    cross-attention bytes per step) are as even as a longest-first greedy gets them. Each
    shard's indices come back in increasing order, and the assignment is deterministic."""
    if world < 1:
        raise ValueError("need world >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    load = [0] * world
    count = [0] * world
    shards: list[list[int]] = [[] for _ in range(world)]
    cap = -(-len(lengths) // world)  # at most ceil(n / world) items per rank (KV arena slots)
    for i in order:
        r = min((r for r in range(world) if count[r] < cap), key=lambda r: (load[r], r))
        shards[r].append(i)
        load[r] += int(lengths[i])
        count[r] += 1
    return [sorted(s) for s in shards]


def max_over_ranks(x: float, group=None) -> float:
    """The largest value of `x` over all ranks (device times of a timed region)."""
    import torch
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(x)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else "cpu"
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def run_sharded(fn: Callable[[list[int]], list], shards: list[list[int]], n: int,
                group=None) -> list | None:
    """Runs fn(this rank's indices) -> one result per index, gathers every rank's results and
    returns them in global index order on rank 0 (None on the other ranks). Every rank must
    call it with the same `shards`. An exception raised by fn on any rank reaches every rank as
    a RuntimeError naming the failed ranks."""
    import torch.distributed as dist
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    if len(shards) != world:
        raise ValueError(f"{len(shards)} shards for {world} ranks")
    mine = shards[rank]
    try:
        res = list(fn(mine))
        if len(res) != len(mine):
            raise RuntimeError(f"rank {rank}: {len(res)} results for {len(mine)} items")
        payload = ("ok", res)
    except Exception as e:  # reported to every rank, then raised everywhere
        payload = ("error", f"rank {rank}: {type(e).__name__}: {e}")
    if world == 1:
        gathered = [payload]
    else:
        gathered = [None] * world
        dist.all_gather_object(gathered, payload, group=group)
    errors = [p[1] for p in gathered if p[0] == "error"]
    if errors:
        raise RuntimeError("sharded run failed: " + "; ".join(errors))
    if rank != 0:
        return None
    out: list = [None] * n
    for r, (_, res) in enumerate(gathered):
        for i, v in zip(shards[r], res):
            out[i] = v
    return out
