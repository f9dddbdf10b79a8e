"""Checkpoint ingestion (bitnetrs_b200.weights and the native conversions
bitnet_cuda_decode_hf_packed, bitnet_cuda_absmean_ternary and
bitnet_cuda_lm_head_i8_table), on CPU.

* the HF packed-lane decode against the known answers transcribed from the
  reference (tests/golden/kats.json, fn "hf_decode") and against the oracle's
  restatement of decode_packed_projection on random tensors;
* absmean ternarisation and the i8 lm_head table against the oracle;
* both loaders end to end through safetensors files written here: a packed
  checkpoint made from a seeded model must load back to exactly that model,
  and a dense checkpoint must load to the oracle's absmean of its values;
* the loaders' errors for missing, misshapen and mistyped tensors.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle_lib as O
from bitnetrs_b200 import InvalidShape, ModelConfig, QuantizationError, synth
from bitnetrs_b200 import weights as Wt
from kat_runner import by_fn, pack_rows

L = O.lib()
ERRORS = {"InvalidShape": InvalidShape, "QuantizationError": QuantizationError}


def _unpack_rows(packed, rows, cols):
    pc = (cols + 3) // 4
    out = np.zeros((rows, cols), dtype=np.int8)
    for r in range(rows):
        row = np.ascontiguousarray(packed[r * pc:(r + 1) * pc])
        assert L.orc_unpack_ternary(O.p(row), pc, cols, O.p(out[r])) == 0
    return out


def _encode_hf(values):
    """Inverse of decode_packed_projection: logical [4*pr][cols] ternary -> HF bytes [pr][cols]."""
    rows, cols = values.shape
    pr = rows // 4
    lanes = (values.astype(np.int16) + 1).astype(np.uint8).reshape(4, pr, cols)
    return (lanes[0] | (lanes[1] << 2) | (lanes[2] << 4) | (lanes[3] << 6)).astype(np.uint8)


@pytest.mark.parametrize("k", by_fn("hf_decode"), ids=lambda k: k["name"])
def test_hf_decode_kats(k):
    pk = np.array(k["packed"], dtype=np.uint8)
    if "error" in k:
        with pytest.raises(ERRORS[k["error"]], match=None if "message" not in k else r"\(1, 3\), shift 4"):
            Wt.decode_hf_packed(pk, k["packed_rows"], k["cols"], k["scale"])
    else:
        out = Wt.decode_hf_packed(pk, k["packed_rows"], k["cols"], k["scale"])
        np.testing.assert_array_equal(out, pack_rows(k["rows"]))


@pytest.mark.parametrize("pr,cols", [(1, 1), (2, 4), (37, 91), (160, 640)])
def test_hf_decode_matches_oracle(pr, cols):
    lanes = synth.uniform_u32(9, pr * 7 + cols, 4 * pr * cols, 0, 2).astype(np.uint8).reshape(4, pr, cols)
    hf = (lanes[0] | (lanes[1] << 2) | (lanes[2] << 4) | (lanes[3] << 6)).astype(np.uint8)
    logical = np.zeros(4 * pr * cols, dtype=np.int8)
    assert L.orc_decode_hf_packed(O.p(hf), hf.size, pr, cols, 0.5, O.p(logical)) == 0
    out = Wt.decode_hf_packed(hf, pr, cols, 0.5)
    np.testing.assert_array_equal(out, pack_rows(logical.reshape(4 * pr, cols).tolist()))
    np.testing.assert_array_equal(_encode_hf(logical.reshape(4 * pr, cols)), hf)


def test_hf_decode_reports_first_bad_lane_in_scan_order():
    hf = np.full((64, 32), 0x55, dtype=np.uint8)
    hf[40, 3] = 0b11_01_01_01  # shift 6
    hf[7, 30] = 0b01_01_11_01  # shift 2, earlier packed row: reported
    with pytest.raises(QuantizationError, match=r"\(7, 30\), shift 2"):
        Wt.decode_hf_packed(hf, 64, 32, 1.0)


@pytest.mark.parametrize("rows,cols", [(1, 1), (13, 70), (64, 257)])
def test_absmean_matches_oracle(rows, cols):
    w = synth.normal_f32(4, rows + cols, rows * cols, std=0.02)
    q = np.zeros(rows * cols, dtype=np.int8)
    s = O.C.c_float()
    assert L.orc_absmean_quantize(O.p(w), w.size, O.p(q), O.C.byref(s)) == 0
    out, scale = Wt.absmean_ternary(w, rows, cols)
    assert np.float32(scale) == np.float32(s.value)
    np.testing.assert_array_equal(out, pack_rows(q.reshape(rows, cols).tolist()))


def test_absmean_errors():
    with pytest.raises(QuantizationError, match="empty"):
        Wt.absmean_ternary(np.zeros(0, np.float32), 0, 4)
    with pytest.raises(QuantizationError, match="index 2"):
        Wt.absmean_ternary(np.array([1.0, 0.5, np.nan, 0.0], np.float32), 1, 4)


def test_lm_head_i8_matches_oracle():
    rows, H = 40, 96
    e = synth.bf16_normal(6, 2, rows * H, 0.02)
    e[5 * H:6 * H] = 0  # all-zero row: minimum scale
    q_ref = np.zeros(rows * H, dtype=np.int8)
    s_ref = np.zeros(rows, dtype=np.float32)
    L.orc_quantize_bf16_rows_to_i8(O.p(e), rows, H, O.p(q_ref), O.p(s_ref))
    q, s = Wt.lm_head_i8(e, rows, H)
    np.testing.assert_array_equal(q, q_ref)
    np.testing.assert_array_equal(s, s_ref)


CFG = ModelConfig(96, 64, 2, 4, 2, 128, 64, 10000.0, 1e-5)


def _packed_checkpoint(w, cfg):
    """A packed checkpoint holding exactly the model `w` (scales stored as F32)."""
    H, F, V, qd, kvd = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.q_dim(), cfg.kv_dim()
    t = {"model.embed_tokens.weight": ("BF16", (V, H), w.embed_tokens),
         "model.norm.weight": ("F32", (H,), w.final_norm)}
    for i, Lw in enumerate(w.layers):
        b = f"model.layers.{i}"
        t[f"{b}.input_layernorm.weight"] = ("F32", (H,), Lw.attention_norm)
        t[f"{b}.post_attention_layernorm.weight"] = ("F32", (H,), Lw.ffn_norm)
        t[f"{b}.self_attn.attn_sub_norm.weight"] = ("F32", (H,), Lw.attn_sub_norm)
        t[f"{b}.mlp.ffn_sub_norm.weight"] = ("F32", (F,), Lw.ffn_sub_norm)
        for name, arr, scale, rows, cols in (("self_attn.q_proj", Lw.q_proj, Lw.q_scale, qd, H),
                                             ("self_attn.k_proj", Lw.k_proj, Lw.k_scale, kvd, H),
                                             ("self_attn.v_proj", Lw.v_proj, Lw.v_scale, kvd, H),
                                             ("self_attn.o_proj", Lw.o_proj, Lw.o_scale, H, qd),
                                             ("mlp.gate_proj", Lw.gate_proj, Lw.gate_scale, F, H),
                                             ("mlp.up_proj", Lw.up_proj, Lw.up_scale, F, H),
                                             ("mlp.down_proj", Lw.down_proj, Lw.down_scale, H, F)):
            hf = _encode_hf(_unpack_rows(arr, rows, cols))
            t[f"{b}.{name}.weight"] = ("U8", hf.shape, hf)
            t[f"{b}.{name}.weight_scale"] = ("F32", (1,), np.array([scale], np.float32))
    return t


def test_packed_checkpoint_loads_back_exactly(tmp_path):
    w = synth.random_model(CFG, seed=13)
    path = tmp_path / "model.safetensors"
    Wt.write_safetensors(path, _packed_checkpoint(w, CFG))
    got = Wt.load_weights_from_packed(path, CFG)
    np.testing.assert_array_equal(got.embed_tokens, w.embed_tokens)
    np.testing.assert_array_equal(got.lm_head_i8, w.lm_head_i8)
    np.testing.assert_array_equal(got.lm_head_scales, w.lm_head_scales)
    np.testing.assert_array_equal(got.final_norm, w.final_norm)
    for a, b in zip(got.layers, w.layers):
        for f in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj", "attention_norm",
                  "attn_sub_norm", "ffn_norm", "ffn_sub_norm"):
            np.testing.assert_array_equal(getattr(a, f), getattr(b, f), err_msg=f)
        for f in ("q_scale", "k_scale", "v_scale", "o_scale", "gate_scale", "up_scale", "down_scale"):
            assert np.float32(getattr(a, f)) == np.float32(getattr(b, f)), f


def test_packed_checkpoint_errors(tmp_path):
    w = synth.random_model(CFG, seed=13)
    base = _packed_checkpoint(w, CFG)

    def load(mut):
        t = dict(base)
        mut(t)
        path = tmp_path / "bad.safetensors"
        Wt.write_safetensors(path, t)
        return Wt.load_weights_from_packed(path, CFG)

    k = "model.layers.1.mlp.down_proj.weight"
    with pytest.raises(InvalidShape, match="missing packed projection tensor"):
        load(lambda t: t.pop(k))
    with pytest.raises(InvalidShape, match="missing scale tensor"):
        load(lambda t: t.pop(k + "_scale"))
    with pytest.raises(InvalidShape, match="expected U8/I8"):
        load(lambda t: t.__setitem__(k, ("F32", (16, 128), np.zeros(16 * 128, np.float32))))
    with pytest.raises(InvalidShape, match="via 4x expansion"):
        load(lambda t: t.__setitem__(k, ("U8", (8, 128), np.zeros(8 * 128, np.uint8))))
    with pytest.raises(InvalidShape, match="columns"):
        load(lambda t: t.__setitem__(k, ("U8", (32, 64), np.zeros(32 * 64, np.uint8))))
    with pytest.raises(InvalidShape, match="missing float tensor 'model.norm.weight'"):
        load(lambda t: t.pop("model.norm.weight"))
    with pytest.raises(QuantizationError, match="weight_scale"):
        load(lambda t: t.__setitem__(k + "_scale", ("F32", (1,), np.array([-1.0], np.float32))))


def test_bf16_checkpoint_absmean_on_load(tmp_path):
    cfg = CFG
    H, F, V, qd, kvd = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.q_dim(), cfg.kv_dim()
    t, dense = {}, {}
    stream = [100]

    def bf16(shape, std):
        stream[0] += 1
        bits = synth.bf16_normal(3, stream[0], int(np.prod(shape)), std)
        return ("BF16", shape, bits)

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
            dense[f"{b}.{n}"] = (rows, cols)
    path = tmp_path / "dense.safetensors"
    Wt.write_safetensors(path, t)
    got = Wt.load_weights_from_bf16(path, cfg)
    np.testing.assert_array_equal(got.embed_tokens, t["model.embed_tokens.weight"][2])
    for i, Lw in enumerate(got.layers):
        b = f"model.layers.{i}"
        for f, n in (("q_proj", "self_attn.q_proj"), ("o_proj", "self_attn.o_proj"), ("down_proj", "mlp.down_proj")):
            rows, cols = dense[f"{b}.{n}"]
            w = (t[f"{b}.{n}.weight"][2].astype(np.uint32) << 16).view(np.float32)
            q = np.zeros(rows * cols, dtype=np.int8)
            s = O.C.c_float()
            assert L.orc_absmean_quantize(O.p(w), w.size, O.p(q), O.C.byref(s)) == 0
            np.testing.assert_array_equal(getattr(Lw, f), pack_rows(q.reshape(rows, cols).tolist()))
            assert np.float32(getattr(Lw, f.replace("_proj", "_scale"))) == np.float32(s.value)
        np.testing.assert_array_equal(Lw.ffn_sub_norm,
                                      (t[f"{b}.mlp.ffn_sub_norm.weight"][2].astype(np.uint32) << 16).view(np.float32))


def test_safetensors_round_trip(tmp_path):
    t = {"a": ("F32", (2, 3), np.arange(6, dtype=np.float32)), "b": ("U8", (5,), np.arange(5, dtype=np.uint8)),
         "c": ("BF16", (4,), np.array([0x3F80, 0, 0xBF80, 0x7FC0], np.uint16))}
    Wt.write_safetensors(tmp_path / "x.safetensors", t)
    r = Wt.read_safetensors(tmp_path / "x.safetensors")
    assert set(r) == {"a", "b", "c"}
    for k, (dt, shp, arr) in t.items():
        assert r[k].dtype == dt and r[k].shape == shp
        np.testing.assert_array_equal(np.asarray(r[k].data), arr)


def test_load_model_config(tmp_path):
    p = tmp_path / "config.json"
    p.write_text('{"vocab_size": 128256, "hidden_size": 2560, "num_hidden_layers": 30, "num_attention_heads": 20,'
                 ' "num_key_value_heads": 5, "intermediate_size": 6912, "max_position_embeddings": 4096,'
                 ' "rope_theta": 500000.0, "rms_norm_eps": 1e-05}')
    from bitnetrs_b200 import bitnet_2b_config

    assert Wt.load_model_config(p) == bitnet_2b_config()
    p.write_text('{"vocab_size": 10, "hidden_size": 8, "num_hidden_layers": 1, "num_attention_heads": 2,'
                 ' "intermediate_size": 16, "max_position_embeddings": 32}')
    c = Wt.load_model_config(p)
    assert c.num_key_value_heads == 2 and c.rope_theta == 10000.0 and c.rms_norm_eps == 1e-5


def test_detect_format_resolve_config_and_load(tmp_path):
    # detect_weight_format (inference/src/lib.rs:428-452), resolve_model_config
    # (lib.rs:455-488, tests lib.rs:1359-1400)
    from bitnetrs_b200 import bitnet_2b_config

    w = synth.random_model(CFG, seed=13)
    d = tmp_path / "m"
    d.mkdir()
    path = d / "model.safetensors"
    Wt.write_safetensors(path, _packed_checkpoint(w, CFG))
    assert Wt.detect_weight_format(path) == "packed"
    assert Wt.resolve_model_config(path) == bitnet_2b_config()  # no sibling config.json
    (d / "config.json").write_text(
        '{"vocab_size": 96, "hidden_size": 64, "num_hidden_layers": 2, "num_attention_heads": 4,'
        ' "num_key_value_heads": 2, "intermediate_size": 128, "max_position_embeddings": 64}')
    assert Wt.resolve_model_config(path) == CFG
    got = Wt.load_weights(path)
    np.testing.assert_array_equal(got.layers[1].down_proj, w.layers[1].down_proj)
    dense = d / "dense.safetensors"
    Wt.write_safetensors(dense, {"x": ("F32", (2,), np.zeros(2, np.float32))})
    assert Wt.detect_weight_format(dense) == "bf16"
    junk = d / "junk.safetensors"
    junk.write_bytes(b"\x00\x01")
    assert Wt.detect_weight_format(junk) == "bf16"
