"""Tensor parallelism for models too large for one GPU: one process per GPU.

The shards and the per-layer collectives live in the native library
(``bitnet_cuda_model_create_tp``): each rank keeps the q/k/v rows of its
heads, the gate/up rows of its intermediate slice and the matching input
columns of o_proj and down_proj, all-gathers the attention output and the
gated FFN activation (both sub-norms then run over full rows, in the
reference's order) and all-reduces the int32 accumulators of o_proj and
down_proj over NCCL. Every rank's hidden state is therefore bit-identical to
the single-GPU model's. This module checks a configuration against the split
rules, describes each rank's share, and agrees on the NCCL id over a
``torch.distributed`` group.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Dict, Tuple

from . import _native as N
from .errors import InvalidConfig

ID_BYTES = 128  # BITNET_TP_ID_BYTES


@dataclass(frozen=True)
class TensorParallel:
    """This process's place in a tensor-parallel group and the group's NCCL id."""

    rank: int
    world: int
    unique_id: bytes


def check_config(cfg, world: int) -> None:
    """Raise InvalidConfig unless `cfg` splits over `world` ranks: query and
    KV heads divisible by world, and each rank's attention width and
    intermediate slice multiples of 64 columns (the same rules, in the same
    order, as bitnet_cuda_model_create_tp)."""
    if world < 1:
        raise InvalidConfig("tensor-parallel rank must be < world (world > 0)")
    nh, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    if nh % world or nkv % world:
        raise InvalidConfig(f"num_attention_heads ({nh}) and num_key_value_heads ({nkv}) must be divisible by the "
                            f"tensor-parallel world ({world})")
    qd = cfg.q_dim()
    F = cfg.intermediate_size
    if F % world or (qd // world) % 64 or (F // world) % 64:
        raise InvalidConfig(f"per-rank attention width ({qd // world}) and intermediate slice ({F // world}) must be "
                            "multiples of 64")


def shard(cfg, rank: int, world: int) -> Dict[str, Tuple[int, int]]:
    """Half-open index ranges owned by `rank`: query heads, KV heads, q/o
    columns, k/v rows, and gate/up rows (= down columns)."""
    check_config(cfg, world)
    if not 0 <= rank < world:
        raise InvalidConfig("tensor-parallel rank must be < world (world > 0)")
    nh, nkv, hd = cfg.num_attention_heads // world, cfg.num_key_value_heads // world, cfg.head_dim()
    f = cfg.intermediate_size // world
    return {
        "q_heads": (rank * nh, (rank + 1) * nh),
        "kv_heads": (rank * nkv, (rank + 1) * nkv),
        "q_cols": (rank * nh * hd, (rank + 1) * nh * hd),
        "kv_rows": (rank * nkv * hd, (rank + 1) * nkv * hd),
        "ffn_rows": (rank * f, (rank + 1) * f),
    }


def unique_id() -> bytes:
    """A fresh NCCL id (made on one rank, shared with the others)."""
    lib = N.cuda_lib()
    buf = (C.c_uint8 * ID_BYTES)()
    N.check(lib.bitnet_cuda_tp_unique_id(buf, ID_BYTES))
    return bytes(buf)


def init(group=None) -> TensorParallel:
    """Rank 0 of the torch.distributed group makes the NCCL id and broadcasts
    it; every rank returns its TensorParallel (rank and world of the group)."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    obj = [unique_id() if rank == 0 else None]
    src = 0 if group is None else dist.get_global_rank(group, 0)
    dist.broadcast_object_list(obj, src=src, group=group)
    return TensorParallel(rank, world, obj[0])
