"""Host logic of tensor parallelism, on CPU.

The split rules (the same checks bitnet_cuda_model_create_tp makes before any
device work), the ownership ranges of each rank, the decomposition the device
path relies on (a row-split projection's int32 sums over column slices add up
to the full sum; sqrelu gating commutes with the all-gather), and agreement
on the NCCL id across two gloo ranks.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from bitnetrs_b200 import InvalidConfig, ModelConfig, bitnet_2b_config, scaled_model_config, synth, tp


def test_scaled_shape_splits_over_1_2_4_8():
    cfg = scaled_model_config()
    assert (cfg.hidden_size, cfg.num_hidden_layers, cfg.num_attention_heads, cfg.num_key_value_heads,
            cfg.intermediate_size) == (4096, 32, 32, 8, 14336)
    for world in (1, 2, 4, 8):
        tp.check_config(cfg, world)


def test_split_rules_reject():
    with pytest.raises(InvalidConfig, match="divisible"):
        tp.check_config(bitnet_2b_config(), 2)  # 5 KV heads
    with pytest.raises(InvalidConfig, match="multiples of 64"):
        tp.check_config(ModelConfig(100, 256, 1, 8, 8, 96, 64, 1e4, 1e-5), 2)  # 48-column FFN slice
    with pytest.raises(InvalidConfig, match="multiples of 64"):
        tp.check_config(ModelConfig(100, 256, 1, 8, 8, 256, 64, 1e4, 1e-5), 8)  # 32-column attention slice
    with pytest.raises(InvalidConfig):
        tp.check_config(scaled_model_config(), 0)
    with pytest.raises(InvalidConfig):
        tp.shard(scaled_model_config(), 8, 8)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shards_partition_and_keep_gqa_groups(world):
    cfg = scaled_model_config()
    group = cfg.num_attention_heads // cfg.num_key_value_heads
    parts = [tp.shard(cfg, r, world) for r in range(world)]
    for key, total in (("q_heads", cfg.num_attention_heads), ("kv_heads", cfg.num_key_value_heads),
                       ("q_cols", cfg.q_dim()), ("kv_rows", cfg.kv_dim()), ("ffn_rows", cfg.intermediate_size)):
        spans = [p[key] for p in parts]
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    for p in parts:
        lo, hi = p["kv_heads"]
        # every query head of the rank reads a KV head the rank holds
        assert all(lo <= h // group < hi for h in range(*p["q_heads"]))


def _codes(packed_row, n):
    b = np.frombuffer(packed_row, dtype=np.uint8)
    c = np.stack([(b >> (2 * j)) & 3 for j in range(4)], axis=1).reshape(-1)[:n]
    return np.where(c == 0, 1, np.where(c == 2, -1, 0)).astype(np.int64)


@pytest.mark.parametrize("world", [2, 4])
def test_row_split_int32_sums_add_up(world):
    # o_proj-like [N, K] in the reference 2-bit format; each rank holds the
    # byte columns [r*K/world/4, (r+1)*K/world/4) of every row
    N, K, M = 48, 512, 5
    packed = synth.ternary_codes(3, 7, N, K).reshape(N, K // 4)
    xq = synth.uniform_u32(3, 8, M * K, 0, 255).astype(np.int64).reshape(M, K) - 128
    W = np.stack([_codes(packed[i].tobytes(), K) for i in range(N)])
    full = xq @ W.T
    k = K // world
    total = np.zeros_like(full)
    for r in range(world):
        cols = packed[:, r * k // 4:(r + 1) * k // 4]
        Wr = np.stack([_codes(cols[i].tobytes(), k) for i in range(N)])
        np.testing.assert_array_equal(Wr, W[:, r * k:(r + 1) * k])
        total += xq[:, r * k:(r + 1) * k] @ Wr.T
    np.testing.assert_array_equal(total, full)
    assert np.abs(full).max() < 2**31


def test_gate_then_gather_equals_gathered_gate():
    T, F, world = 3, 256, 4
    rng = np.random.default_rng(5)
    g = rng.standard_normal((T, F)).astype(np.float32)
    u = rng.standard_normal((T, F)).astype(np.float32)

    def gate(a, b):
        r = np.maximum(a, np.float32(0))
        return (r * r) * b

    f = F // world
    chunks = [gate(g[:, r * f:(r + 1) * f], u[:, r * f:(r + 1) * f]) for r in range(world)]
    gathered = np.stack(chunks)  # [world][T][f], what an all-gather returns
    rows = gathered.transpose(1, 0, 2).reshape(T, F)  # the unchunk re-layout
    np.testing.assert_array_equal(rows, gate(g, u))


def test_unique_id_bytes():
    a, b = tp.unique_id(), tp.unique_id()
    assert len(a) == tp.ID_BYTES == 128 and len(b) == 128


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        t = tp.init()
        out.put((rank, t.rank, t.world, t.unique_id))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_share_one_id():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = sorted(q.get(timeout=120) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert [g[0] for g in got] == [0, 1] and [g[1] for g in got] == [0, 1]
    assert all(g[2] == 2 for g in got)
    assert got[0][3] == got[1][3] and len(got[0][3]) == 128
