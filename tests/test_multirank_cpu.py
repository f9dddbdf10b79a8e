"""Host logic of multi-GPU data-parallel decode, on CPU ranks (gloo).

Two gloo ranks place a request list with dp.shard_requests, each decodes its
own share greedily with the CPU oracle (the checker the GPU tests use), and
rank 0 checks that the union equals a single-process decode of every
request, that the shares partition the list and balance KV work, and that
the max-over-ranks reduction returns the slowest rank's value.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from bitnetrs_b200 import ModelConfig, dp, synth


def test_shard_requests_equal_counts_and_balance():
    import numpy as np

    rng = np.random.default_rng(3)
    for world in (1, 2, 4, 8):
        ctx = rng.integers(128, 4097, size=256 * world).tolist()
        shards = dp.shard_requests_equal(ctx, world, 256)
        assert sorted(i for s in shards for i in s) == list(range(len(ctx)))
        assert all(len(s) == 256 for s in shards)
        loads = dp.shard_loads(ctx, shards)
        assert max(loads) - min(loads) <= max(ctx) + 1
        assert dp.shard_requests_equal(ctx, world, 256) == shards
    assert dp.shard_requests_equal(list(range(6)), 1, 6) == [list(range(6))]
    with pytest.raises(ValueError):
        dp.shard_requests_equal([1, 2, 3], 2, 2)


def test_shard_requests_partition_and_balance():
    ctx = synth.uniform_u32(3, 11, 256, 128, 4096).astype(np.int64)
    for world in (1, 2, 4, 8):
        shards = dp.shard_requests(ctx, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(len(ctx)))
        loads = dp.shard_loads(ctx, shards)
        # LPT bound: max load <= mean + largest item
        assert max(loads) <= sum(loads) / world + int(ctx.max()) + 1
        assert dp.shard_requests(ctx, world) == shards  # deterministic
    assert dp.shard_requests([], 3) == [[], [], []]
    with pytest.raises(ValueError):
        dp.shard_requests([1, 2], 0)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


CFG = ModelConfig(300, 64, 2, 4, 2, 96, 128, 10000.0, 1e-5)
PROMPTS = [[(7 * i + 3 * j) % CFG.vocab_size for j in range(2 + (5 * i) % 9)] for i in range(6)]
NEW = 5


def _decode(indices):
    import oracle_lib as O

    w = synth.random_model(CFG, seed=4)
    om = O.OracleModel(w)
    out = {}
    for i in indices:
        kv = om.kv(CFG.max_position_embeddings)
        toks, _ = om.generate(kv, PROMPTS[i], NEW, eos=(CFG.vocab_size + 1, CFG.vocab_size + 2))
        out[i] = toks
    return out


def _rank(rank, world, port, q):
    import sys

    import torch.distributed as dist

    here = os.path.dirname(os.path.abspath(__file__))
    for p in (here, os.path.dirname(here)):
        if p not in sys.path:
            sys.path.insert(0, p)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        shards = dp.shard_requests([len(p) for p in PROMPTS], world)
        mine = _decode(shards[rank])
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        slowest = dp.max_over_ranks(10.0 + rank)
        if rank == 0:
            merged = {}
            for g in gathered:
                merged.update(g)
            q.put((shards, merged, slowest))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_decode_their_shares():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        shards, merged, slowest = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    assert sorted(merged) == list(range(len(PROMPTS)))
    assert all(shards)  # both ranks got work
    assert slowest == 11.0
    single = _decode(range(len(PROMPTS)))
    assert merged == single
