"""The device sampler (bitnet_cuda_sample_next_token, generate_sampled)
against the oracle's restatement of sample_next_token
(crates/bitnet-inference/src/lib.rs:236-390): the reference's sampler tests
(tests/golden/kats.json, fn "sample"), then random logits over many seeds
and configurations at the test vocabulary and at the 2B vocabulary (128256),
with the logits the reference modifies in place compared too, and a sampled
generation through the model against the oracle's forward + sampler loop.
Tokens must be identical."""
import numpy as np
import pytest

import oracle_lib as O
from bitnetrs_b200 import BackendError, BitNetModel, InvalidConfig, KV_BF16, ModelConfig, synth
from bitnetrs_b200.sampling import SamplingConfig
from kat_runner import by_fn, f

pytestmark = pytest.mark.gpu
L = O.lib()


def oracle_sample(logits, cfg, past=()):
    lg = np.array(logits, dtype=np.float32)
    pa = np.ascontiguousarray(np.asarray(past, dtype=np.uint32))
    tok = int(L.orc_sample_next_token(O.p(lg), lg.size, cfg.temperature, cfg.top_p, cfg.top_k,
                                      cfg.repetition_penalty, cfg.seed, O.p(pa) if pa.size else None, pa.size))
    return tok, lg


def cfg_of(d, seed=None):
    return SamplingConfig(d["temperature"], d["top_p"], d["top_k"], d["repetition_penalty"], 1,
                          d["seed"] if seed is None else seed)


@pytest.mark.parametrize("k", by_fn("sample"), ids=lambda k: k["name"])
def test_sampler_kats(cuda_backend, k):
    logits = np.array(f(k["logits"]), dtype=np.float32)
    if "token" in k:
        assert cuda_backend.sample_next_token(logits.copy(), cfg_of(k["cfg"]), k["past"]) == k["token"]
    else:
        for seed in range(k.get("seeds", 1)):
            c = cfg_of(k["cfg"], seed if "seeds" in k else None)
            tok = cuda_backend.sample_next_token(logits.copy(), c, k["past"])
            assert tok in k["allowed"], (seed, tok)
            assert tok == oracle_sample(logits, c, k["past"])[0]


CONFIGS = [
    SamplingConfig.chat_defaults(),                       # t 0.7, top-p 0.9, top-k 50, penalty 1.1
    SamplingConfig(1.0, 0.95, 200, 1.05, 1, 0),
    SamplingConfig(1.3, 0.5, 4000, 1.0, 1, 0),
    SamplingConfig(0.9, 1.0, 0, 1.2, 1, 0),               # whole vocabulary, no top-p: the streamed path
    SamplingConfig(1.0, 1.0, 10, 1.0, 1, 0),
    SamplingConfig(0.5, 1.0, 1, 1.3, 1, 0),               # greedy shortcut after penalty and temperature
]


@pytest.mark.parametrize("vocab", [1000, 128256])
@pytest.mark.parametrize("ci", range(len(CONFIGS)))
def test_sampler_matches_oracle(cuda_backend, vocab, ci):
    base = CONFIGS[ci]
    rng = np.random.default_rng(1000 * ci + vocab)
    for trial in range(6):
        logits = (rng.standard_normal(vocab) * rng.uniform(0.5, 4.0)).astype(np.float32)
        past = rng.integers(0, vocab, size=int(rng.integers(0, 300))).astype(np.uint32)
        if past.size:
            past[: past.size // 3] = past[0]  # a repeated token: one division per occurrence
        c = base.with_(seed=int(rng.integers(0, 2**63)))
        got_logits = logits.copy()
        tok = cuda_backend.sample_next_token(got_logits, c, past)
        ref, ref_logits = oracle_sample(logits, c, past)
        assert tok == ref, (trial, tok, ref)
        np.testing.assert_array_equal(got_logits, ref_logits)


def test_sampler_large_nucleus_is_reported(cuda_backend):
    logits = np.zeros(128256, dtype=np.float32)
    with pytest.raises(BackendError, match="4096"):
        cuda_backend.sample_next_token(logits, SamplingConfig(1.0, 0.9, 0, 1.0, 1, 0))


def test_generate_sampled_matches_oracle(cuda_backend):
    cfg = ModelConfig(1000, 512, 2, 4, 1, 768, 256, 500000.0, 1e-5)
    w = synth.random_model(cfg, seed=23)
    m = BitNetModel(w, cuda_backend, max_batch_tokens=64)
    kv = m.new_kv_cache(num_pages=32, kv_dtype=KV_BF16)
    om = O.OracleModel(w)
    prompt = synth.uniform_u32(8, 2, 21, 0, cfg.vocab_size - 1).tolist()
    for sc in (SamplingConfig.chat_defaults().with_(seed=7), SamplingConfig(1.1, 1.0, 0, 1.05, 1, 3)):
        got = m.generate(kv, prompt, 20, sampling=sc)
        okv = om.kv(cfg.max_position_embeddings, bf16=True)
        lg = om.forward(okv, prompt, 0)
        toks, ref = list(prompt), []
        for _ in range(20):
            t, _ = oracle_sample(lg, sc, toks)
            if t in (128009, 128001):
                break
            ref.append(t)
            toks.append(t)
            lg = om.forward(okv, [t], len(toks) - 1)
        assert got == ref
    with pytest.raises(InvalidConfig):
        m.generate(kv, prompt, 4, sampling=SamplingConfig(0.0, 0.9, 50, 1.1, 1, 0))
    kv.close()
    m.close()
