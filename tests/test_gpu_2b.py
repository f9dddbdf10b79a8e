"""Parity at the benchmarked 2B shape (hidden 2560, 30 layers, 20/5 heads of
128, FFN 6912, vocab 128256), random init, against the CPU oracle's
BitNetModel::forward:

* C1: a 128-token seeded prompt and 128 greedy steps at batch 1, in the
  default (reference-order) numerics with f32 and bf16 caches, and the
  measured deviation of FAST numerics (tensor-core attention and lm_head);
* C4: one batch-256 decode step over seeded contexts U[128, 4096], the
  configuration bench.py times, with sampled rows decoded by the oracle.

The GPU is fed the oracle's tokens (teacher forcing) so every step compares
logits on identical inputs.  Tolerances: reference-order numerics are
bit-identical; the tensor-core lm_head of many-row steps sums in a different
order (at hidden 2560, within 5e-5 of the largest logit); FAST does not meet the north-star 1e-2
at this shape, and its test records by how much."""
import dataclasses

import numpy as np
import pytest

import oracle_lib as O
from bitnetrs_b200 import KV_BF16, KV_F32, BitNetModel, bitnet_2b_config, synth

pytestmark = pytest.mark.gpu

CTX_LO, CTX_HI = 128, 4096


@pytest.fixture(scope="module")
def w2b():
    cfg = bitnet_2b_config()
    cfg = dataclasses.replace(cfg, max_position_embeddings=CTX_HI + 64)
    return synth.random_model(cfg, seed=0)


@pytest.fixture(scope="module")
def oracle2b(w2b):
    return O.OracleModel(w2b)


def _c1_run(cuda_backend, w, om, kv_dtype, mode):
    cfg = w.config
    prompt = synth.uniform_u32(0, 2, 128, 0, cfg.vocab_size - 1).tolist()
    m = BitNetModel(w, cuda_backend, max_batch_tokens=256)
    m.set_numerics(mode)
    kv = m.new_kv_cache(num_pages=32, kv_dtype=kv_dtype)
    okv = om.kv(512, bf16=(kv_dtype == KV_BF16))
    L = O.lib()
    g = m.forward(prompt, 0, kv)
    r = om.forward(okv, prompt, 0)
    stats = []
    for step in range(128):
        tok = int(L.orc_greedy_argmax(O.p(r), r.size))
        top2 = np.partition(r, -2)[-2:]
        margin = float(top2[1] - top2[0])
        err = float(np.max(np.abs(g - r)))
        gtok = int(cuda_backend.greedy_argmax(g))
        stats.append((step, err, margin, tok, gtok, float(np.max(np.abs(r)))))
        pos = len(prompt) + step
        g = m.forward([tok], pos, kv)
        r = om.forward(okv, [tok], pos)
    kv.close()
    m.close()
    return stats


@pytest.mark.parametrize("kv_dtype", [KV_F32, KV_BF16], ids=["f32kv", "bf16kv"])
def test_2b_greedy_decode_token_identical(cuda_backend, w2b, oracle2b, kv_dtype):
    """C1 in the default numerics: logits bit-identical to the oracle at
    every one of 128 steps, so every greedy token is identical."""
    stats = _c1_run(cuda_backend, w2b, oracle2b, kv_dtype, "auto")
    errs = np.array([s[1] for s in stats])
    bad = [s[:5] for s in stats if s[3] != s[4]]
    print(f"max |dlogit| {errs.max():.3g}; bit-identical steps {int(np.sum(errs == 0))}/128; "
          f"min oracle top-2 margin {min(s[2] for s in stats):.3g}; token mismatches {bad}")
    assert not bad, f"greedy token differs at {bad[:3]} (step, |dlogit|, oracle top-2 margin, ref, gpu)"
    assert int(np.sum(errs == 0)) == 128


def test_2b_fast_numerics_deviation(cuda_backend, w2b, oracle2b):
    """C1 in FAST numerics (tensor-core attention at every size).  FAST does
    NOT meet the north-star 1e-2 bound at the 2B shape: the tensor-core
    attention rounds differently from the reference, the next int8
    quantisation amplifies each difference, and over 30 layers the logits
    move by ~10% of the largest logit (measured on a B200: max 0.125, with 22
    of 128 greedy tokens different).  This test pins that characterisation so
    a regression shows: logits within 0.2 of the largest logit and at least
    two thirds of the greedy tokens equal.  The default numerics, which the
    benchmark runs, are bit-identical (test above)."""
    stats = _c1_run(cuda_backend, w2b, oracle2b, KV_BF16, "fast")
    worst = max(s[1] / s[5] for s in stats)
    flips = [s[:5] for s in stats if s[3] != s[4]]
    print(f"FAST: max relative |dlogit| {worst:.3g}; {len(flips)} token mismatches {flips}")
    assert worst <= 0.2
    assert len(flips) <= len(stats) // 3


def test_2b_batch256_decode_sampled_rows(cuda_backend, w2b, oracle2b):
    """C4 as bench.py runs it: 256 sequences with seeded contexts U[128,
    4096] (the bench's seed), one decode step and a second on the GPU's
    tokens, in the default numerics (tcgen05 GEMM, reference-order TMA
    attention, tcgen05 lm_head).  Six sampled rows (spread over the batch,
    plus the longest context) are decoded by the oracle from the same bf16
    contexts.  Every hidden state is bit-exact; the lm_head's f32 sums over
    2560 products run in the tensor core's order, measured at 1.0e-5 to
    1.2e-5 of the largest logit, so logits are held to 5e-5 of it and greedy
    tokens must be equal wherever the top-2 margin exceeds 1e-4 of it."""
    cfg = w2b.config
    B = 256
    ctxs = synth.uniform_u32(0, 11, B, CTX_LO, CTX_HI).astype(np.int64)
    rows = sorted({0, 64, 128, 192, 255, int(np.argmax(ctxs))})
    m = BitNetModel(w2b, cuda_backend, max_batch_tokens=B)
    kv = m.new_kv_cache(num_pages=int(np.sum((ctxs + 4 + 15) // 16)) + 16, max_seqs=B, kv_dtype=KV_BF16)
    host = {}
    for i in range(B):
        if i in rows:
            host[i] = synth.kv_normal(0, i, cfg, int(ctxs[i]))
            kv.write(i, *host[i])
        else:
            kv.fill_random(i, int(ctxs[i]), 0)
    assert m.attention_kernel(kv, B) == "attn_qk_softmax_kernel+attn_pv_kernel"
    toks = synth.uniform_u32(0, 3, B, 0, cfg.vocab_size - 1)
    seqs = list(range(B))
    steps = []
    for _ in range(2):
        nxt, logits = m.decode_step(kv, seqs, toks, want_logits=True)
        steps.append((toks[rows].copy(), nxt[rows].copy(), logits[rows].copy()))
        del logits
        toks = nxt
    kv.close()
    m.close()
    L = O.lib()
    report = []
    for j, i in enumerate(rows):
        okv = oracle2b.kv(int(ctxs[i]) + 4, bf16=True)
        okv.seed(*host.pop(i))
        for s, (tin, tout, lg) in enumerate(steps):
            r = oracle2b.forward(okv, [int(tin[j])], int(ctxs[i]) + s)
            scale = float(np.max(np.abs(r)))
            err = float(np.max(np.abs(lg[j] - r)))
            top2 = np.partition(r, -2)[-2:]
            ref_tok = int(L.orc_greedy_argmax(O.p(r), r.size))
            report.append((i, int(ctxs[i]), s, err / scale, ref_tok, int(tout[j])))
            assert err <= 5e-5 * scale, f"row {i} (context {ctxs[i]}) step {s}: |dlogit| {err} vs max {scale}"
            if top2[1] - top2[0] > 1e-4 * scale:
                assert int(tout[j]) == ref_tok, f"row {i} step {s}: token {tout[j]} vs oracle {ref_tok}"
        del okv
    print("row, context, step, rel |dlogit|, oracle token, gpu token:", report)


def test_2b_ragged_prefill_packed(cuda_backend, w2b, oracle2b):
    """C3 as bench.py runs it, at a size the oracle finishes in seconds: five
    seeded prompts of lengths U[32, 300] packed into steps of at most 512
    tokens (bitnetrs_b200.batching.pack_steps; a prompt continues in the next
    step), bf16 paged cache, default numerics (tcgen05 GEMM at M up to 512,
    reference-order causal attention).  Each prompt's last logits and greedy
    token must equal the oracle's forward over the same prompt: fewer than 17
    output rows per step keep the lm_head in reference order, so the logits
    are bit-identical."""
    cfg = w2b.config
    lens = synth.uniform_u32(0, 21, 5, 32, 300).astype(int).tolist()
    prompts = [synth.uniform_u32(0, 100 + s, n, 0, cfg.vocab_size - 1) for s, n in enumerate(lens)]
    m = BitNetModel(w2b, cuda_backend, max_batch_tokens=512)
    kv = m.new_kv_cache(num_pages=sum((n + 15) // 16 for n in lens) + 16, max_seqs=len(lens), kv_dtype=KV_BF16)
    nxt, logits = m.prefill_packed(kv, list(range(len(lens))), prompts, want_logits=True)
    kv.close()
    m.close()
    assert sum(lens) > 512  # at least two steps, one prompt split across them
    L = O.lib()
    for i, p in enumerate(prompts):
        okv = oracle2b.kv(lens[i] + 4, bf16=True)
        r = oracle2b.forward(okv, p.tolist(), 0)
        np.testing.assert_array_equal(logits[i], r, err_msg=f"prompt {i} (length {lens[i]})")
        assert int(nxt[i]) == int(L.orc_greedy_argmax(O.p(r), r.size))
        del okv
