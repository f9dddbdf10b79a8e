"""Packing of ragged prompts into prefill steps (bitnetrs_b200.batching): every
step fits the model's token capacity, each sequence appears at most once per
step, and each prompt's chunks cover it exactly once, in order."""
import numpy as np
import pytest

from bitnetrs_b200.batching import pack_steps


def check_packing(lengths, cap):
    steps = pack_steps(lengths, cap)
    seen = {i: 0 for i in range(len(lengths))}
    for st in steps:
        assert 0 < sum(c for _, _, c in st) <= cap
        idx = [i for i, _, _ in st]
        assert len(idx) == len(set(idx)), "a sequence twice in one step"
        for i, a, c in st:
            assert c > 0 and a == seen[i], "chunks out of order or overlapping"
            seen[i] += c
    assert all(seen[i] == n for i, n in enumerate(lengths))
    # steps are full except possibly the last
    assert all(sum(c for _, _, c in st) == cap for st in steps[:-1])
    return steps


@pytest.mark.parametrize("cap", [1, 4, 16, 64, 1024])
def test_random_ragged(cap):
    rng = np.random.default_rng(cap)
    for _ in range(50):
        lens = rng.integers(0, 3 * cap + 5, size=int(rng.integers(0, 12))).tolist()
        check_packing(lens, cap)


def test_edges():
    assert pack_steps([], 8) == []
    assert pack_steps([0, 0], 8) == []
    assert pack_steps([8], 8) == [[(0, 0, 8)]]
    assert pack_steps([9], 8) == [[(0, 0, 8)], [(0, 8, 1)]]
    assert pack_steps([3, 5, 2], 8) == [[(0, 0, 3), (1, 0, 5)], [(2, 0, 2)]]
    with pytest.raises(ValueError):
        pack_steps([1], 0)
    with pytest.raises(ValueError):
        pack_steps([-1], 4)
