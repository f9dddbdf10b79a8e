"""Host-side packing of ragged prompts into prefill steps.

``bitnet_cuda_prefill`` runs one step of at most the model's token capacity
(``max_batch_tokens``). A serving loop with more prompt tokens than that packs
them into consecutive steps: prompts are taken in order, a step is filled up
to the capacity, and a prompt that does not fit continues at the start of the
next step. Each sequence therefore appears at most once per step, and its
chunks arrive in order, so every token sees exactly the context the reference
gives it when the prompt is run token by token (the per-sequence math of
``BitNetModel::forward``, crates/bitnet-model/src/lib.rs:559-862).
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

Chunk = Tuple[int, int, int]  # (index into the prompt list, first token, token count)


def pack_steps(lengths: Sequence[int], max_tokens: int) -> List[List[Chunk]]:
    """Split prompts of the given lengths into steps of at most ``max_tokens`` tokens.

    Returns one list of (prompt index, start, count) chunks per step. Empty
    prompts contribute no chunk."""
    if max_tokens < 1:
        raise ValueError("max_tokens must be at least 1")
    steps: List[List[Chunk]] = []
    cur: List[Chunk] = []
    used = 0
    for i, n in enumerate(lengths):
        if n < 0:
            raise ValueError(f"prompt {i} has negative length {n}")
        pos = 0
        while pos < n:
            take = min(n - pos, max_tokens - used)
            cur.append((i, pos, take))
            pos += take
            used += take
            if used == max_tokens:
                steps.append(cur)
                cur, used = [], 0
    if cur:
        steps.append(cur)
    return steps
