"""Tensor-parallel model shards against the single-device model.

A shard's hidden state is bit-identical to the single-device model's by
construction (both sub-norms run over all-gathered full rows, the o_proj and
down_proj accumulators are summed exactly in int32), so logits and greedy
tokens must be equal, not close. The script covers the three matmul paths:
an 84-token ragged prefill (tensor-core GEMM), 3-sequence decode steps and a
single-token forward (GEMV). World 1 runs the whole tensor-parallel path (an
NCCL communicator of one rank, the row split, re-layout and epilogue kernels)
on one GPU; world 2 needs two GPUs.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from bitnetrs_b200 import KV_BF16, BitNetModel, CudaBackend, InvalidConfig, ModelConfig, synth, tp

pytestmark = pytest.mark.gpu

# head_dim 128, 4 query / 2 KV heads, FFN 768: splits over 1 and 2 ranks
CFG = ModelConfig(1000, 512, 2, 4, 2, 768, 256, 10000.0, 1e-5)
SEED = 21
PROMPTS = [[(11 * i + 7 * j) % CFG.vocab_size for j in range(n)] for i, n in enumerate((5, 70, 9))]


def _script(model):
    kv = model.new_kv_cache(num_pages=64, max_seqs=3, kv_dtype=KV_BF16)
    out = []
    nxt, lg = model.prefill(kv, [0, 1, 2], PROMPTS, want_logits=True)
    out += [lg, nxt]
    for _ in range(4):
        nxt, lg = model.decode_step(kv, [0, 1, 2], nxt, want_logits=True)
        out += [lg, nxt]
    out.append(model.forward([int(nxt[0])], kv.len(0), kv, seq=0))
    kv.close()
    return out


@pytest.fixture(scope="module")
def weights():
    return synth.random_model(CFG, seed=SEED)


def test_tp_world1_bit_identical(cuda_backend, weights):
    ref = BitNetModel(weights, cuda_backend, max_batch_tokens=128)
    want = _script(ref)
    ref.close()
    m = BitNetModel(weights, cuda_backend, max_batch_tokens=128, tp=tp.TensorParallel(0, 1, tp.unique_id()))
    got = _script(m)
    m.close()
    assert len(got) == len(want)
    for a, b in zip(got, want):
        np.testing.assert_array_equal(a, b)


def test_tp_rejects_bad_split(cuda_backend, weights):
    uid = tp.unique_id()
    with pytest.raises(InvalidConfig, match="divisible"):
        BitNetModel(weights, cuda_backend, max_batch_tokens=16, tp=tp.TensorParallel(0, 3, uid))
    with pytest.raises(InvalidConfig, match="rank must be < world"):
        BitNetModel(weights, cuda_backend, max_batch_tokens=16, tp=tp.TensorParallel(2, 2, uid))


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _tp_rank(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        t = tp.init()
        be = CudaBackend(rank)
        w = synth.random_model(CFG, seed=SEED)
        m = BitNetModel(w, be, max_batch_tokens=128, tp=t)
        got = _script(m)
        m.close()
        if rank == 0:
            ref = BitNetModel(w, be, max_batch_tokens=128)
            want = _script(ref)
            ref.close()
            same = len(got) == len(want) and all(np.array_equal(a, b) for a, b in zip(got, want))
            out.put((rank, same))
        else:
            out.put((rank, True))
    except Exception as e:  # reported to the parent, which fails the test
        out.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp_world2_bit_identical():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = sorted(q.get(timeout=300) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert got == [(0, True), (1, True)], got
