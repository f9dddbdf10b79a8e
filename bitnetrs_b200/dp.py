"""Data-parallel request placement for batched decode across GPUs.

Sequences are independent, so a node serves a request list by giving each
rank (one process per GPU, weights replicated) a subset and running no
collective on the data path.  Decode time is dominated by reading each
sequence's KV cache, so subsets are balanced by KV bytes -- the context
length of each sequence -- with the longest-processing-time-first greedy
rule, not by request count.  Every rank computes the same placement from the
same inputs, so no message is needed to agree on it.
"""
from __future__ import annotations

from typing import List, Sequence


def shard_requests(ctx_lens: Sequence[int], world: int) -> List[List[int]]:
    """Split request indices over `world` ranks, balancing sum(ctx_len + 1).

    Requests are taken longest first and each goes to the rank with the least
    load so far (ties to the lower rank); each rank's indices come back in
    ascending order.  Deterministic for equal inputs.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(ctx_lens)), key=lambda i: (-(int(ctx_lens[i]) + 1), i))
    load = [0] * world
    out: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += int(ctx_lens[i]) + 1
    return [sorted(s) for s in out]


def shard_requests_equal(ctx_lens: Sequence[int], world: int, per_rank: int) -> List[List[int]]:
    """Split `world * per_rank` requests into `world` sets of exactly
    `per_rank`, balancing sum(ctx_len + 1) with the same longest-first greedy
    rule as :func:`shard_requests`, restricted to ranks that still have room.
    This is the placement for a fixed batch per GPU (weak scaling): every
    rank decodes the same number of sequences and about the same KV bytes."""
    if world < 1 or per_rank < 0:
        raise ValueError("world must be >= 1 and per_rank >= 0")
    if len(ctx_lens) != world * per_rank:
        raise ValueError("expected world * per_rank requests")
    order = sorted(range(len(ctx_lens)), key=lambda i: (-(int(ctx_lens[i]) + 1), i))
    load = [0] * world
    out: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min((k for k in range(world) if len(out[k]) < per_rank), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += int(ctx_lens[i]) + 1
    return [sorted(s) for s in out]


def shard_loads(ctx_lens: Sequence[int], shards: List[List[int]]) -> List[int]:
    """KV positions each rank reads per decode step."""
    return [sum(int(ctx_lens[i]) + 1 for i in s) for s in shards]


def max_over_ranks(value: float, device=None) -> float:
    """Largest `value` over the ranks of the default process group (the
    whole-job time of a step is the slowest rank's); identity when no group
    is initialised."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
