"""Checkpoint ingestion end to end on the GPU: a seeded model written as a
packed HF checkpoint (the reference's load_weights_from_packed path,
crates/bitnet-weights/src/loader.rs:523 via decode_packed_projection,
crates/bitnet-convert/src/lib.rs:235-317) and a dense bf16 checkpoint
(load_weights_from_bf16, loader.rs:396-490, absmean on load), each with a
sibling config.json, loaded through bitnetrs_b200.weights.load_weights
(format detection and config resolution as the engine does), uploaded to
the device and run: the prompt's logits are bit-identical to the oracle's
BitNetModel::forward on the same loaded weights, and greedy generation gives
the same tokens.  The model has head_dim 128 and a GQA group of 4, so the
step runs the tcgen05 GEMM, the reference-order QK/PV attention kernels
and the tensor-core lm_head where the batch allows."""
import json

import numpy as np
import pytest

import oracle_lib as O
from bitnetrs_b200 import KV_BF16, BitNetModel, ModelConfig, synth
from bitnetrs_b200 import weights as Wt
from test_weights_cpu import _packed_checkpoint

pytestmark = pytest.mark.gpu

CFG = ModelConfig(1000, 512, 2, 4, 1, 768, 256, 500000.0, 1e-5)


def _config_json(d, cfg):
    (d / "config.json").write_text(json.dumps({
        "vocab_size": cfg.vocab_size, "hidden_size": cfg.hidden_size, "num_hidden_layers": cfg.num_hidden_layers,
        "num_attention_heads": cfg.num_attention_heads, "num_key_value_heads": cfg.num_key_value_heads,
        "intermediate_size": cfg.intermediate_size, "max_position_embeddings": cfg.max_position_embeddings,
        "rope_theta": cfg.rope_theta, "rms_norm_eps": cfg.rms_norm_eps}))


def _dense_checkpoint(cfg, seed):
    H, F, V, qd, kvd = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.q_dim(), cfg.kv_dim()
    t = {}
    stream = [200]

    def bf16(shape, std):
        stream[0] += 1
        return ("BF16", shape, synth.bf16_normal(seed, stream[0], int(np.prod(shape)), std))

    t["model.embed_tokens.weight"] = bf16((V, H), 0.02)
    t["model.norm.weight"] = bf16((H,), 1.0)
    for i in range(cfg.num_hidden_layers):
        b = f"model.layers.{i}"
        for n, shp in (("input_layernorm", (H,)), ("post_attention_layernorm", (H,)),
                       ("self_attn.attn_sub_norm", (H,)), ("mlp.ffn_sub_norm", (F,))):
            t[f"{b}.{n}.weight"] = bf16(shp, 1.0)
        for n, rows, cols in (("self_attn.q_proj", qd, H), ("self_attn.k_proj", kvd, H), ("self_attn.v_proj", kvd, H),
                              ("self_attn.o_proj", H, qd), ("mlp.gate_proj", F, H), ("mlp.up_proj", F, H),
                              ("mlp.down_proj", H, F)):
            t[f"{b}.{n}.weight"] = bf16((rows, cols), 0.02)
    return t


def _run_and_compare(cuda_backend, w, prompt):
    m = BitNetModel(w, cuda_backend, max_batch_tokens=128)
    kv = m.new_kv_cache(num_pages=32, kv_dtype=KV_BF16)
    om = O.OracleModel(w)
    okv = om.kv(w.config.max_position_embeddings, bf16=True)
    np.testing.assert_array_equal(m.forward(prompt, 0, kv), om.forward(okv, prompt, 0))
    kv.close()
    kv = m.new_kv_cache(num_pages=32, kv_dtype=KV_BF16)
    got = m.generate(kv, prompt, 24)
    ref, _ = om.generate(om.kv(w.config.max_position_embeddings, bf16=True), prompt, 24)
    assert got == ref
    kv.close()
    m.close()


def test_packed_checkpoint_runs_on_gpu(cuda_backend, tmp_path):
    w = synth.random_model(CFG, seed=17)
    Wt.write_safetensors(tmp_path / "model.safetensors", _packed_checkpoint(w, CFG))
    _config_json(tmp_path, CFG)
    path = tmp_path / "model.safetensors"
    assert Wt.detect_weight_format(path) == "packed"
    loaded = Wt.load_weights(path)
    assert loaded.config == CFG
    np.testing.assert_array_equal(loaded.layers[1].gate_proj, w.layers[1].gate_proj)
    _run_and_compare(cuda_backend, loaded, synth.uniform_u32(4, 1, 37, 0, CFG.vocab_size - 1).tolist())


def test_bf16_checkpoint_runs_on_gpu(cuda_backend, tmp_path):
    Wt.write_safetensors(tmp_path / "model.safetensors", _dense_checkpoint(CFG, seed=5))
    _config_json(tmp_path, CFG)
    path = tmp_path / "model.safetensors"
    assert Wt.detect_weight_format(path) == "bf16"
    loaded = Wt.load_weights(path)
    assert loaded.config == CFG
    _run_and_compare(cuda_backend, loaded, synth.uniform_u32(6, 1, 29, 0, CFG.vocab_size - 1).tolist())
