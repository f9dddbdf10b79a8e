"""The one-token decode kernel (decode1_kernel: every layer of a batch-1 step
in one persistent launch) against the per-layer kernels, which the other GPU
tests hold bit-identical to the oracle's BitNetModel::forward
(crates/bitnet-model/src/lib.rs:559-860).  The fused kernel performs the same
operations in the same order, so logits must be equal, not close.

Covered: GQA groups 1, 2, 4 and 8; contexts from the first position to
3000+ positions (the attention CTAs' page ring then refills many times per
layer, and pages of a layer run ahead into the next); the eager forward path
and the captured decode-step graph; a one-token forward against the oracle
directly; and the kernel choice itself (bf16 caches only, FAST numerics and
the per-layer switch fall back)."""
import numpy as np
import pytest

import oracle_lib as O
from bitnetrs_b200 import KV_BF16, KV_F32, BitNetModel, ModelConfig, synth

pytestmark = pytest.mark.gpu

CFGS = {
    "gq4": ModelConfig(1000, 512, 2, 4, 1, 768, 4096, 500000.0, 1e-5),
    "gq2": ModelConfig(1000, 512, 2, 4, 2, 768, 4096, 10000.0, 1e-5),
    "gq1": ModelConfig(1000, 256, 3, 2, 2, 512, 4096, 10000.0, 1e-5),
    "gq8": ModelConfig(1000, 1024, 2, 8, 1, 1536, 4096, 10000.0, 1e-5),
}


@pytest.fixture(scope="module", params=sorted(CFGS))
def weights(request):
    return synth.random_model(CFGS[request.param], seed=31)


def _run(m, ctx0, steps, seed):
    """Logits of `steps` one-token forwards after a random context of ctx0
    positions (or a 9-token prompt when ctx0 == 0)."""
    V = m.config.vocab_size
    kv = m.new_kv_cache(num_pages=(ctx0 + steps + 32) // 16 + 2, kv_dtype=KV_BF16)
    if ctx0:
        kv.fill_random(0, ctx0, seed)
        pos = ctx0
        lg = None
    else:
        prompt = [(7 * i + 3) % V for i in range(9)]
        lg = m.forward(prompt, 0, kv)
        pos = len(prompt)
    out = []
    tok = 5
    for _ in range(steps):
        lg = m.forward([tok], pos, kv)
        out.append(lg)
        tok = int(np.argmax(lg))
        pos += 1
    assert m.attention_kernel(kv, 1) == "decode1_kernel"
    kv.close()
    return out


@pytest.mark.parametrize("ctx0,steps", [(0, 6), (40, 3), (3000, 3)])
def test_fused_equals_per_layer(cuda_backend, weights, ctx0, steps):
    m = BitNetModel(weights, cuda_backend, max_batch_tokens=64)
    got = _run(m, ctx0, steps, 17)
    m.set_fused_decode(False)
    kv = m.new_kv_cache(num_pages=4, kv_dtype=KV_BF16)
    assert m.attention_kernel(kv, 1) != "decode1_kernel"
    kv.close()
    want = []
    V = m.config.vocab_size
    kv = m.new_kv_cache(num_pages=(ctx0 + steps + 32) // 16 + 2, kv_dtype=KV_BF16)
    if ctx0:
        kv.fill_random(0, ctx0, 17)
        pos = ctx0
    else:
        prompt = [(7 * i + 3) % V for i in range(9)]
        m.forward(prompt, 0, kv)
        pos = len(prompt)
    tok = 5
    for _ in range(steps):
        lg = m.forward([tok], pos, kv)
        want.append(lg)
        tok = int(np.argmax(lg))
        pos += 1
    kv.close()
    m.close()
    for i, (a, b) in enumerate(zip(got, want)):
        np.testing.assert_array_equal(a, b, err_msg=f"step {i}")


def test_fused_decode_graph_steps(cuda_backend):
    """decode_step at batch 1 (the captured graph, sized for the cache's
    capacity) equals the per-layer graph, tokens and logits, over 24 steps
    that cross page boundaries; greedy generate agrees too."""
    w = synth.random_model(CFGS["gq4"], seed=5)
    res = []
    for fused in (True, False):
        m = BitNetModel(w, cuda_backend, max_batch_tokens=64)
        m.set_fused_decode(fused)
        kv = m.new_kv_cache(num_pages=16, kv_dtype=KV_BF16)
        nxt, lg0 = m.prefill(kv, [0], [[11, 12, 13, 14, 15, 16, 17]], want_logits=True)
        toks, lgs = [int(nxt[0])], [lg0]
        for _ in range(24):
            nxt, lg = m.decode_step(kv, [0], [toks[-1]], want_logits=True)
            toks.append(int(nxt[0]))
            lgs.append(lg)
        kv.close()
        kv = m.new_kv_cache(num_pages=16, kv_dtype=KV_BF16)
        gen = m.generate(kv, [11, 12, 13, 14, 15, 16, 17], 20)
        kv.close()
        m.close()
        res.append((toks, lgs, gen))
    (t1, l1, g1), (t2, l2, g2) = res
    assert t1 == t2
    assert g1 == g2 == t1[:20]
    for a, b in zip(l1, l2):
        np.testing.assert_array_equal(a, b)


def test_fused_one_token_forward_matches_oracle(cuda_backend):
    """The fused step on its own against the oracle: a prompt, then one-token
    forwards, logits bit-identical (bf16 cache on both sides)."""
    cfg = CFGS["gq2"]
    w = synth.random_model(cfg, seed=8)
    om = O.OracleModel(w)
    m = BitNetModel(w, cuda_backend, max_batch_tokens=64)
    kv = m.new_kv_cache(num_pages=8, kv_dtype=KV_BF16)
    okv = om.kv(128, bf16=True)
    prompt = [3, 1, 4, 1, 5, 9, 2, 6]
    g = m.forward(prompt, 0, kv)
    r = om.forward(okv, prompt, 0)
    np.testing.assert_array_equal(g, r)
    for step in range(12):
        tok = int(np.argmax(r))
        pos = len(prompt) + step
        g = m.forward([tok], pos, kv)
        r = om.forward(okv, [tok], pos)
        np.testing.assert_array_equal(g, r, err_msg=f"step {step}")
    assert m.attention_kernel(kv, 1) == "decode1_kernel"
    kv.close()
    m.close()


def test_fused_kernel_choice(cuda_backend):
    """f32 caches and FAST numerics keep the per-layer kernels; multi-token
    steps never use the fused kernel."""
    w = synth.random_model(CFGS["gq4"], seed=6)
    m = BitNetModel(w, cuda_backend, max_batch_tokens=64)
    kv16 = m.new_kv_cache(num_pages=8, kv_dtype=KV_BF16)
    kv32 = m.new_kv_cache(num_pages=8, kv_dtype=KV_F32)
    assert m.attention_kernel(kv16, 1) == "decode1_kernel"
    assert m.attention_kernel(kv16, 2) != "decode1_kernel"
    assert m.attention_kernel(kv32, 1) != "decode1_kernel"
    m.set_numerics("fast")
    assert m.attention_kernel(kv16, 1) != "decode1_kernel"
    m.set_numerics("exact")
    assert m.attention_kernel(kv16, 1) == "decode1_kernel"
    kv16.close()
    kv32.close()
    m.close()
