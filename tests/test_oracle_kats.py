"""Pins the CPU oracle (restatement of the reference CPU backend) against the
known-answer vectors transcribed from the reference's unit tests, plus exact
numpy restatements of its integer paths.  CPU only."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib as O
from kat_runner import KATS, by_fn, f, pack_rows

L = O.lib()
p = O.p


def err(rc):
    return O.ERR[rc]


def test_host_has_avx2_fma():
    assert L.orc_has_avx2_fma() == 1


@pytest.mark.parametrize("k", by_fn("pack"), ids=lambda k: k["name"])
def test_pack(k):
    vals = np.array(k["values"], dtype=np.int8)
    out = np.zeros((vals.size + 3) // 4, dtype=np.uint8)
    L.orc_pack_ternary(p(vals), vals.size, p(out))
    if "packed" in k:
        assert out.tolist() == k["packed"]
    if "packed_len" in k:
        assert out.size == k["packed_len"]
    if k.get("roundtrip"):
        back = np.zeros(vals.size, dtype=np.int8)
        assert L.orc_unpack_ternary(p(out), out.size, vals.size, p(back)) == 0
        assert back.tolist() == k["values"]


@pytest.mark.parametrize("k", by_fn("unpack"), ids=lambda k: k["name"])
def test_unpack_errors(k):
    pk = np.array(k["packed"], dtype=np.uint8)
    out = np.zeros(k["n"], dtype=np.int8)
    assert err(L.orc_unpack_ternary(p(pk), pk.size, k["n"], p(out))) == k["error"]


@pytest.mark.parametrize("k", by_fn("hf_decode"), ids=lambda k: k["name"])
def test_hf_decode(k):
    pk = np.array(k["packed"], dtype=np.uint8)
    out = np.zeros(max(4 * k["packed_rows"] * k["cols"], 1), dtype=np.int8)
    rc = L.orc_decode_hf_packed(p(pk), pk.size, k["packed_rows"], k["cols"], k["scale"], p(out))
    if "error" in k:
        assert err(rc) == k["error"]
    else:
        assert rc == 0
        assert out.reshape(-1, k["cols"]).tolist() == k["rows"]


def test_packed_bytes_row_aligned():
    (k,) = by_fn("packed_bytes")
    for rows, cols, expected in k["cases"]:
        assert rows * ((cols + 3) // 4) == expected


@pytest.mark.parametrize("k", by_fn("absmax"), ids=lambda k: k["name"])
def test_absmax(k):
    x = f(k["x"])
    q = np.zeros(x.size, dtype=np.int8)
    s = C.c_float()
    rc = L.orc_absmax_quantize_row_into(p(x), x.size, p(q), q.size, C.byref(s))
    if "error" in k:
        assert err(rc) == k["error"]
        return
    assert rc == 0
    if "q" in k:
        assert q.tolist() == k["q"]
    for i, v in k.get("q_at", {}).items():
        assert q[int(i)] == v
    if "scale" in k:
        assert abs(s.value - k["scale"]) <= k["scale_tol"] + 1e-12
    if k.get("scale_positive"):
        assert s.value > 0


@pytest.mark.parametrize("k", by_fn("absmean"), ids=lambda k: k["name"])
def test_absmean(k):
    w = f(k["w"])
    q = np.zeros(max(1, w.size), dtype=np.int8)
    s = C.c_float()
    rc = L.orc_absmean_quantize(p(w), w.size, p(q), C.byref(s))
    if "error" in k:
        assert err(rc) == k["error"]
        return
    assert rc == 0
    assert q[: w.size].tolist() == k["q"]
    if "scale" in k:
        assert abs(s.value - k["scale"]) <= k["scale_tol"] + 1e-12


@pytest.mark.parametrize("k", by_fn("gemv_f32"), ids=lambda k: k["name"])
def test_gemv_f32(k):
    w = pack_rows(k["w"])
    x = f(k["x"])
    N, K = len(k["w"]), len(k["w"][0])
    out = np.full(N, 7.0, dtype=np.float32)
    assert L.orc_ternary_gemv(p(w), w.size, k["scale"], p(x), x.size, p(out), out.size, N, K) == 0
    np.testing.assert_allclose(out, k["out"], atol=k["tol"], rtol=0)


@pytest.mark.parametrize("k", by_fn("gemv_f32_raw"), ids=lambda k: k["name"])
def test_gemv_f32_errors(k):
    w = np.zeros(k["packed_len"], dtype=np.uint8)
    x = np.zeros(k["x_len"], dtype=np.float32)
    out = np.zeros(k["out_len"], dtype=np.float32)
    assert err(L.orc_ternary_gemv(p(w), w.size, k["scale"], p(x), x.size, p(out), out.size, k["N"], k["K"])) == k[
        "error"]


@pytest.mark.parametrize("k", by_fn("dot_i8"), ids=lambda k: k["name"])
def test_dot_i8(k):
    w = pack_rows([k["w"]])
    x = np.array(k["x"], dtype=np.int8)
    out = np.zeros(1, dtype=np.float32)
    acc = np.zeros(1, dtype=np.int32)
    assert L.orc_ternary_gemv_preq(p(w), w.size, 1.0, p(x), x.size, 127.0, p(out), 1, 1, x.size, p(acc)) == 0
    assert acc[0] == k["acc"]
    assert out[0] == np.float32(k["acc"])  # combined = 1*127/127 = 1


@pytest.mark.parametrize("k", by_fn("gemv_q_formula"), ids=lambda k: k["name"])
def test_gemv_quantised_formula(k):
    w = f(k["w"])
    q = np.zeros(w.size, dtype=np.int8)
    ws = C.c_float()
    assert L.orc_absmean_quantize(p(w), w.size, p(q), C.byref(ws)) == 0
    x = f(k["x"])
    xq = np.zeros(x.size, dtype=np.int8)
    xs = C.c_float()
    assert L.orc_absmax_quantize_row_into(p(x), x.size, p(xq), xq.size, C.byref(xs)) == 0
    rows, cols = k["rows"], k["cols"]
    packed = pack_rows(q.reshape(rows, cols).tolist())
    out = np.zeros(rows, dtype=np.float32)
    max_abs = np.float32(xs.value) * np.float32(127.0)
    assert L.orc_ternary_gemv_preq(p(packed), packed.size, ws.value, p(xq), xq.size, float(max_abs), p(out), rows,
                                   rows, cols, None) == 0
    for r in range(rows):
        acc = int(np.dot(q.reshape(rows, cols)[r].astype(np.int32), xq.astype(np.int32)))
        # the reference test's own expectation formula (gemv.rs:593-607 / :648)
        act = xs.value if k["expect"] == "acc*ws*x_scale/127" else max_abs
        exp = np.float32(acc) * np.float32(ws.value) * np.float32(act) / np.float32(127.0)
        assert abs(out[r] - exp) < k["tol"]


def test_gemv_quantised_bad_act_scale():
    (k,) = by_fn("gemv_q_raw")
    w = pack_rows(k["w"])
    xq = np.array(k["xq"], dtype=np.int8)
    out = np.zeros(1, dtype=np.float32)
    assert err(L.orc_ternary_gemv_preq(p(w), w.size, k["scale"], p(xq), xq.size, k["act_absmax"], p(out), 1, 1,
                                       xq.size, None)) == k["error"]


@pytest.mark.parametrize("k", by_fn("rms_norm"), ids=lambda k: k["name"])
def test_rms_norm(k):
    x, w = f(k["x"]), f(k["w"])
    out = np.full(x.size, 99.0, dtype=np.float32)
    rc = L.orc_rms_norm(p(x), x.size, p(w), w.size, k["eps"], p(out), out.size)
    if "error" in k:
        assert err(rc) == k["error"]
        return
    assert rc == 0
    if "out" in k:
        np.testing.assert_allclose(out, k["out"], atol=k["tol"], rtol=0)
    for i, v in k.get("out_at", {}).items():
        assert abs(out[int(i)] - v) < k["tol"]


@pytest.mark.parametrize("k", by_fn("rope"), ids=lambda k: k["name"])
def test_rope(k):
    q, kk = f(k["q"]), f(k["k"])
    rc = L.orc_rope_embed(p(q), q.size, p(kk), kk.size, k["pos"], k["head_dim"], k["n_heads"], k["n_kv_heads"],
                          k["theta"])
    if "error" in k:
        assert err(rc) == k["error"]
        return
    assert rc == 0
    np.testing.assert_allclose(q, k["q_out"], atol=k["tol"], rtol=0)
    np.testing.assert_allclose(kk, k["k_out"], atol=k["tol"], rtol=0)


@pytest.mark.parametrize("k", by_fn("attention"), ids=lambda k: k["name"])
def test_attention(k):
    q, kc, vc = f(k["q"]), f(k["k"]), f(k["v"])
    out = np.zeros(k["n_heads"] * k["head_dim"], dtype=np.float32)
    rc = L.orc_masked_attention(p(q), q.size, p(kc), kc.size, p(vc), vc.size, p(out), out.size, k["n_heads"],
                                k["n_kv_heads"], k["head_dim"], k["cur_pos"])
    if "error" in k:
        assert err(rc) == k["error"]
        return
    assert rc == 0
    np.testing.assert_allclose(out, k["out"], atol=k["tol"], rtol=0)


@pytest.mark.parametrize("k", by_fn("argmax"), ids=lambda k: k["name"])
def test_argmax(k):
    x = f(k["logits"])
    assert L.orc_greedy_argmax(p(x), x.size) == k["token"]


@pytest.mark.parametrize("k", by_fn("tiny_model"), ids=lambda k: k["name"])
def test_tiny_model_golden_logits(k):
    from bitnetrs_b200 import tiny_config
    from bitnetrs_b200.synth import tiny_reference_model

    w = tiny_reference_model(tiny_config())
    m = O.OracleModel(w)
    kv = m.kv(32)
    logits = m.forward(kv, k["tokens"], 0)
    np.testing.assert_allclose(logits, k["logits"], atol=k["tol"], rtol=0)
    assert len(kv) == len(k["tokens"])


# ---------------------------------------------------------------------------
# Exact restatements (numpy) of the oracle's integer / reduction-order paths.
# ---------------------------------------------------------------------------
def unpack(packed, rows, cols):
    pc = (cols + 3) // 4
    b = packed.reshape(rows, pc)
    codes = np.stack([(b >> (2 * j)) & 3 for j in range(4)], axis=-1).reshape(rows, pc * 4)[:, :cols]
    return np.where(codes == 0, 1, np.where(codes == 2, -1, 0)).astype(np.int32)


@pytest.mark.parametrize("N,K", [(7, 13), (64, 2560), (33, 6912), (1, 1)])
def test_oracle_gemv_int32_exact(N, K):
    rng = np.random.default_rng(N * 1000 + K)
    packed = rng.integers(0, 256, size=N * ((K + 3) // 4), dtype=np.uint8)  # includes invalid code 3
    xq = rng.integers(-128, 128, size=K, dtype=np.int8)
    acc = np.zeros(N, dtype=np.int32)
    out = np.zeros(N, dtype=np.float32)
    assert L.orc_ternary_gemv_preq(p(packed), packed.size, 0.0123, p(xq), K, 3.5, p(out), N, N, K, p(acc)) == 0
    W = unpack(packed, N, K)
    np.testing.assert_array_equal(acc, W @ xq.astype(np.int32))
    comb = np.float32(np.float32(0.0123) * np.float32(3.5)) / np.float32(127.0)
    np.testing.assert_array_equal(out, acc.astype(np.float32) * comb)


def rms_norm_ref_order(x, w, eps):
    """norm.rs:113-137 with simd.rs:802-826 order: 8 FMA lanes, hsum, scalar tail."""
    x = x.astype(np.float32)
    d = x.size
    ch = d // 8
    acc = np.zeros(8, dtype=np.float64)
    accf = np.zeros(8, dtype=np.float32)
    for i in range(ch):
        v = x[8 * i: 8 * i + 8].astype(np.float64)
        accf = (v * v + accf.astype(np.float64)).astype(np.float32)  # fma: exact product + one rounding
    del acc
    s = [np.float32(accf[j] + accf[j + 4]) for j in range(4)]
    r = np.float32(np.float32(s[0] + s[1]) + np.float32(s[2] + s[3]))
    for i in range(ch * 8, d):
        r = np.float32(r + np.float32(x[i] * x[i]))
    rms = np.float32(np.sqrt(np.float32(np.float32(r / np.float32(d)) + np.float32(eps))))
    inv = np.float32(np.float32(1.0) / rms)
    return (x * inv).astype(np.float32) * w.astype(np.float32)


@pytest.mark.parametrize("d", [4, 8, 13, 2560, 6912])
def test_oracle_rms_norm_order(d):
    rng = np.random.default_rng(d)
    x = rng.standard_normal(d).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    out = np.zeros(d, dtype=np.float32)
    assert L.orc_rms_norm(p(x), d, p(w), d, 1e-5, p(out), d) == 0
    np.testing.assert_array_equal(out, rms_norm_ref_order(x, w, 1e-5))


def test_oracle_prefill_equals_token_serial():
    """The reference prefill is token-serial (model/src/lib.rs:621-826): a
    multi-token forward equals feeding the tokens one at a time."""
    from bitnetrs_b200 import ModelConfig
    from bitnetrs_b200.synth import random_model

    cfg = ModelConfig(64, 32, 2, 4, 2, 48, 64, 10000.0, 1e-5)
    w = random_model(cfg, seed=3)
    m = O.OracleModel(w)
    toks = [5, 17, 2, 33, 60, 1]
    kv1 = m.kv(64)
    a = m.forward(kv1, toks, 0)
    kv2 = m.kv(64)
    for i, t in enumerate(toks):
        b = m.forward(kv2, [t], i)
    np.testing.assert_array_equal(a, b)
