"""The full sampler's semantics, on CPU: the oracle's restatement of
sample_next_token (crates/bitnet-inference/src/lib.rs:236-390) against the
reference's sampler tests (tests/golden/kats.json, fn "sample", and the
property tests below, which the reference states over sine-wave logits), and
SamplingConfig's presets and validation (fn "sampling_config")."""
from __future__ import annotations

import numpy as np
import pytest

import oracle_lib as O
from bitnetrs_b200 import InvalidConfig
from bitnetrs_b200.sampling import SamplingConfig
from kat_runner import by_fn, f

L = O.lib()


def sample(logits, cfg, past=(), seed=None):
    lg = np.array(logits, dtype=np.float32)
    pa = np.ascontiguousarray(np.asarray(past, dtype=np.uint32))
    s = cfg["seed"] if seed is None else seed
    return int(L.orc_sample_next_token(O.p(lg), lg.size, cfg["temperature"], cfg["top_p"], cfg["top_k"],
                                       cfg["repetition_penalty"], s, O.p(pa) if pa.size else None, pa.size))


def as_dict(c: SamplingConfig):
    return dict(temperature=c.temperature, top_p=c.top_p, top_k=c.top_k, repetition_penalty=c.repetition_penalty,
                seed=c.seed)


@pytest.mark.parametrize("k", by_fn("sample"), ids=lambda k: k["name"])
def test_sample_kats(k):
    logits = f(k["logits"])
    if "token" in k:
        assert sample(logits, k["cfg"], k["past"]) == k["token"]
    else:
        for seed in range(k.get("seeds", 1)):
            tok = sample(logits, k["cfg"], k["past"], seed=seed if "seeds" in k else None)
            assert tok in k["allowed"], (seed, tok)


def test_sample_deterministic_for_same_seed():
    # lib.rs:1172-1193
    cfg = dict(temperature=1.0, top_p=0.9, top_k=10, repetition_penalty=1.0, seed=12345)
    logits = np.sin(np.arange(128, dtype=np.float32) * np.float32(0.17))
    assert sample(logits, cfg) == sample(logits, cfg)


def test_sample_different_seeds_differ():
    # lib.rs:1196-1223
    logits = np.sin(np.arange(128, dtype=np.float32) * np.float32(0.1))
    seen = {sample(logits, dict(temperature=1.5, top_p=1.0, top_k=0, repetition_penalty=1.0, seed=s))
            for s in range(20)}
    assert len(seen) >= 2


def test_sample_stress_in_range():
    # lib.rs:1326-1355: 100 steps over vocab 1024 with the chat-style config
    # and the growing history as the repetition-penalty set
    V = 1024
    gen = []
    for step in range(100):
        i = np.arange(V, dtype=np.float32)
        logits = np.sin(i * np.float32(0.01) + np.float32(step) * np.float32(0.1)) * np.float32(3.0)
        cfg = dict(temperature=0.7, top_p=0.9, top_k=50, repetition_penalty=1.1, seed=42 + step)
        tok = sample(logits, cfg, gen)
        assert 0 <= tok < V
        gen.append(tok)
    assert len(set(gen)) > 1


def test_sample_top_p_keeps_the_nucleus():
    # top_p alone: every draw lies in the smallest prefix (by probability) whose
    # cumulative mass reaches p
    logits = np.array([3.0, 2.0, 1.0, 0.0, -1.0, -2.0], np.float32)
    p = np.exp(logits - logits.max())
    p /= p.sum()
    nucleus = {0, 1}  # 0.63 + 0.23 >= 0.8
    assert p[0] < 0.8 <= p[0] + p[1]
    for s in range(64):
        assert sample(logits, dict(temperature=1.0, top_p=0.8, top_k=0, repetition_penalty=1.0, seed=s)) in nucleus


def test_sample_lcg_draw():
    # one LCG step on seed + len(past) (lib.rs:378-386): uniform logits over 4
    # tokens select floor(u * 4) up to rounding at the bucket edges
    for seed in range(32):
        for n_past in (0, 3):
            st = (seed + n_past) & (2**64 - 1)
            st = (st * 6364136223846793005 + 1442695040888963407) & (2**64 - 1)
            u = float(np.float32(st >> 11) / np.float32(2**53))
            tok = sample(np.zeros(4, np.float32), dict(temperature=1.0, top_p=1.0, top_k=0, repetition_penalty=1.0,
                                                       seed=seed), past=[9] * n_past)
            assert tok == min(int(u * 4), 3) or abs(u * 4 - round(u * 4)) < 1e-6


def test_sampling_config_kats():
    (k,) = by_fn("sampling_config")
    presets = {"greedy": SamplingConfig.greedy(), "chat_defaults": SamplingConfig.chat_defaults(),
               "creative": SamplingConfig.creative(), "default": SamplingConfig()}
    for name in k["valid"]:
        presets[name].validate()
    for change in k["invalid"]:
        with pytest.raises(InvalidConfig):
            SamplingConfig.greedy().with_(**change).validate()
    assert SamplingConfig() == SamplingConfig.chat_defaults()
    assert SamplingConfig.greedy() != SamplingConfig.creative()
    assert SamplingConfig.greedy().is_greedy() and not SamplingConfig.creative().is_greedy()
    # the greedy preset samples the argmax, the other presets are valid draws
    logits = np.array([0.1, 0.5, 5.0, 0.2, -1.0], np.float32)
    assert sample(logits, as_dict(SamplingConfig.greedy())) == 2
