"""Parity at the C5 shape (hidden 4096, 32 layers, 32/8 heads of 128, FFN
14336, vocab 128256) on one GPU, against the CPU oracle's
BitNetModel::forward: the widths the tensor-parallel benchmark runs, through
the single-device kernels (16384-wide norm rows, the tcgen05 GEMM at K =
14336, the batch attention at GQA 4).  Four sequences are prefilled
(ragged, one packed step) and decoded for three steps as a batch; every
step's logits of every sequence must equal the oracle's bit for bit (fewer
than 17 output rows keep the lm_head in reference order)."""
import dataclasses

import numpy as np
import pytest

import oracle_lib as O
from bitnetrs_b200 import KV_BF16, BitNetModel, scaled_model_config, synth

pytestmark = pytest.mark.gpu

LENS = [17, 40, 5, 64]
STEPS = 3


def test_scaled_shape_prefill_and_batched_decode(cuda_backend):
    cfg = dataclasses.replace(scaled_model_config(), max_position_embeddings=256)
    w = synth.random_model_iid(cfg, seed=3)
    prompts = [synth.uniform_u32(3, 50 + s, n, 0, cfg.vocab_size - 1) for s, n in enumerate(LENS)]
    m = BitNetModel(w, cuda_backend, max_batch_tokens=256)
    kv = m.new_kv_cache(num_pages=64, max_seqs=len(LENS), kv_dtype=KV_BF16)
    seqs = list(range(len(LENS)))
    nxt, lg = m.prefill_packed(kv, seqs, prompts, want_logits=True)
    gpu = [(None, lg.copy(), nxt.copy())]
    for _ in range(STEPS):
        inp = nxt
        nxt, lg = m.decode_step(kv, seqs, inp, want_logits=True)
        gpu.append((inp.copy(), lg.copy(), nxt.copy()))
    kv.close()
    m.close()
    om = O.OracleModel(w)
    L = O.lib()
    for i, p in enumerate(prompts):
        okv = om.kv(LENS[i] + STEPS + 2, bf16=True)
        r = om.forward(okv, p.tolist(), 0)
        for s, (inp, lgs, toks) in enumerate(gpu):
            if s > 0:
                r = om.forward(okv, [int(inp[i])], LENS[i] + s - 1)
            np.testing.assert_array_equal(lgs[i], r, err_msg=f"sequence {i} step {s}")
            assert int(toks[i]) == int(L.orc_greedy_argmax(O.p(r), r.size))
        del okv
