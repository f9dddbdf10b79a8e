"""Op-level parity of the CUDA backend (through the C ABI) against the CPU
oracle and the reference's known-answer vectors.

Every op is bit-exact, attention and softmax included (their exp reproduces
the host libm's expf, see ExpTable in csrc/common.cuh)."""
import numpy as np
import pytest

import oracle_lib as O
from bitnetrs_b200 import InvalidConfig, InvalidShape, QuantizationError
from kat_runner import by_fn, f, pack_rows

pytestmark = pytest.mark.gpu
L = O.lib()
p = O.p

ERRS = {"InvalidShape": InvalidShape, "QuantizationError": QuantizationError, "InvalidConfig": InvalidConfig}


# ---------------------------------------------------------------------------
# Known-answer vectors through the CUDA backend
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("k", by_fn("absmax"), ids=lambda k: k["name"])
def test_kat_absmax(cuda_backend, k):
    x = f(k["x"])
    q = np.zeros(x.size, dtype=np.int8)
    if "error" in k:
        with pytest.raises(ERRS[k["error"]]):
            cuda_backend.absmax_quantize_row_into(x, q)
        return
    s = cuda_backend.absmax_quantize_row_into(x, q)
    if "q" in k:
        assert q.tolist() == k["q"]
    for i, v in k.get("q_at", {}).items():
        assert q[int(i)] == v
    if "scale" in k:
        assert abs(s - k["scale"]) <= k["scale_tol"] + 1e-12


@pytest.mark.parametrize("k", by_fn("gemv_f32"), ids=lambda k: k["name"])
def test_kat_gemv_f32(cuda_backend, k):
    w = pack_rows(k["w"])
    x = f(k["x"])
    N, K = len(k["w"]), len(k["w"][0])
    out = np.full(N, 7.0, dtype=np.float32)
    cuda_backend.ternary_gemv(w, k["scale"], x, out, N, K)
    np.testing.assert_allclose(out, k["out"], atol=k["tol"], rtol=0)


@pytest.mark.parametrize("k", by_fn("gemv_f32_raw"), ids=lambda k: k["name"])
def test_kat_gemv_errors(cuda_backend, k):
    w = np.zeros(k["packed_len"], dtype=np.uint8)
    x = np.zeros(k["x_len"], dtype=np.float32)
    out = np.zeros(k["out_len"], dtype=np.float32)
    with pytest.raises(ERRS[k["error"]]):
        cuda_backend.ternary_gemv(w, k["scale"], x, out, k["N"], k["K"])


@pytest.mark.parametrize("k", by_fn("dot_i8"), ids=lambda k: k["name"])
def test_kat_dot_i8(cuda_backend, k):
    w = pack_rows([k["w"]])
    x = np.array(k["x"], dtype=np.int8)
    out = np.zeros(1, dtype=np.float32)
    acc = np.zeros(1, dtype=np.int32)
    cuda_backend.ternary_gemv_preq(w, 1.0, x, 127.0, out, 1, x.size, acc=acc)
    assert acc[0] == k["acc"]
    assert out[0] == np.float32(k["acc"])


def test_kat_gemv_q_bad_act_scale(cuda_backend):
    (k,) = by_fn("gemv_q_raw")
    w = pack_rows(k["w"])
    with pytest.raises(QuantizationError):
        cuda_backend.ternary_gemv_preq(w, k["scale"], np.array(k["xq"], dtype=np.int8), k["act_absmax"],
                                       np.zeros(1, dtype=np.float32), 1, 4)


@pytest.mark.parametrize("k", by_fn("rms_norm"), ids=lambda k: k["name"])
def test_kat_rms_norm(cuda_backend, k):
    x, w = f(k["x"]), f(k["w"])
    out = np.full(x.size, 99.0, dtype=np.float32)
    if "error" in k:
        with pytest.raises(ERRS[k["error"]]):
            cuda_backend.rms_norm(x, w, k["eps"], out)
        return
    cuda_backend.rms_norm(x, w, k["eps"], out)
    if "out" in k:
        np.testing.assert_allclose(out, k["out"], atol=k["tol"], rtol=0)
    for i, v in k.get("out_at", {}).items():
        assert abs(out[int(i)] - v) < k["tol"]


@pytest.mark.parametrize("k", by_fn("rope"), ids=lambda k: k["name"])
def test_kat_rope(cuda_backend, k):
    q, kk = f(k["q"]), f(k["k"])
    if "error" in k:
        with pytest.raises(ERRS[k["error"]]):
            cuda_backend.rope_embed(q, kk, k["pos"], k["head_dim"], k["n_heads"], k["n_kv_heads"], k["theta"])
        return
    cuda_backend.rope_embed(q, kk, k["pos"], k["head_dim"], k["n_heads"], k["n_kv_heads"], k["theta"])
    np.testing.assert_allclose(q, k["q_out"], atol=k["tol"], rtol=0)
    np.testing.assert_allclose(kk, k["k_out"], atol=k["tol"], rtol=0)


@pytest.mark.parametrize("k", by_fn("attention"), ids=lambda k: k["name"])
def test_kat_attention(cuda_backend, k):
    q, kc, vc = f(k["q"]), f(k["k"]), f(k["v"])
    out = np.zeros(k["n_heads"] * k["head_dim"], dtype=np.float32)
    if "error" in k:
        with pytest.raises(ERRS[k["error"]]):
            cuda_backend.masked_attention(q, kc, vc, out, k["n_heads"], k["n_kv_heads"], k["head_dim"], k["cur_pos"])
        return
    cuda_backend.masked_attention(q, kc, vc, out, k["n_heads"], k["n_kv_heads"], k["head_dim"], k["cur_pos"])
    np.testing.assert_allclose(out, k["out"], atol=k["tol"], rtol=0)


@pytest.mark.parametrize("k", by_fn("argmax"), ids=lambda k: k["name"])
def test_kat_argmax(cuda_backend, k):
    assert cuda_backend.greedy_argmax(f(k["logits"])) == k["token"]


# ---------------------------------------------------------------------------
# Seeded random parity against the oracle
# ---------------------------------------------------------------------------
SHAPES = [(2560, 2560), (640, 2560), (6912, 2560), (2560, 6912), (7, 13), (1, 1), (33, 100), (5, 64), (3, 130)]


@pytest.mark.parametrize("N,K", SHAPES)
def test_gemv_preq_int32_and_f32_bit_exact(cuda_backend, N, K):
    rng = np.random.default_rng(N * 7919 + K)
    w = rng.integers(0, 256, size=N * ((K + 3) // 4), dtype=np.uint8)  # includes the invalid code 0b11
    xq = rng.integers(-128, 128, size=K, dtype=np.int8)
    xq[: min(K, 8)] = -128
    ws, amax = np.float32(0.0161), np.float32(3.73)
    acc_o = np.zeros(N, dtype=np.int32)
    out_o = np.zeros(N, dtype=np.float32)
    assert L.orc_ternary_gemv_preq(p(w), w.size, ws, p(xq), K, amax, p(out_o), N, N, K, p(acc_o)) == 0
    acc = np.zeros(N, dtype=np.int32)
    out = np.zeros(N, dtype=np.float32)
    cuda_backend.ternary_gemv_preq(w, ws, xq, amax, out, N, K, acc=acc)
    np.testing.assert_array_equal(acc, acc_o)
    np.testing.assert_array_equal(out, out_o)


@pytest.mark.parametrize("N,K", [(2560, 2560), (2560, 6912), (9, 37), (1, 5)])
def test_gemv_with_activation_quant_bit_exact(cuda_backend, N, K):
    rng = np.random.default_rng(K)
    w = rng.integers(0, 256, size=N * ((K + 3) // 4), dtype=np.uint8)
    x = (rng.standard_normal(K) * 3).astype(np.float32)
    out_o = np.zeros(N, dtype=np.float32)
    assert L.orc_ternary_gemv_with_activation_quant(p(w), w.size, 0.02, p(x), K, p(out_o), N, N, K) == 0
    out = np.zeros(N, dtype=np.float32)
    cuda_backend.ternary_gemv_with_activation_quant(w, 0.02, x, out, N, K)
    np.testing.assert_array_equal(out, out_o)


def test_gemv_with_activation_quant_errors(cuda_backend):
    w = np.zeros(4, dtype=np.uint8)
    out = np.zeros(4, dtype=np.float32)
    with pytest.raises(QuantizationError):  # non-finite input (absmax.rs:148-157)
        cuda_backend.ternary_gemv_with_activation_quant(w, 1.0, np.array([1.0, np.nan, 0, 0], np.float32), out, 4, 4)
    with pytest.raises(QuantizationError):  # input length != in_features reported by the quantiser first
        cuda_backend.ternary_gemv_with_activation_quant(w, 1.0, np.ones(3, np.float32), out, 4, 4)
    with pytest.raises(InvalidShape):
        cuda_backend.ternary_gemv_with_activation_quant(np.zeros(3, np.uint8), 1.0, np.ones(4, np.float32), out, 4, 4)


@pytest.mark.parametrize("N,K", [(2560, 2560), (64, 100), (3, 31)])
def test_gemv_f32_bit_exact(cuda_backend, N, K):
    rng = np.random.default_rng(N + K)
    w = rng.integers(0, 256, size=N * ((K + 3) // 4), dtype=np.uint8)
    x = rng.standard_normal(K).astype(np.float32)
    out_o = np.zeros(N, dtype=np.float32)
    assert L.orc_ternary_gemv(p(w), w.size, 0.37, p(x), K, p(out_o), N, N, K) == 0
    out = np.zeros(N, dtype=np.float32)
    cuda_backend.ternary_gemv(w, 0.37, x, out, N, K)
    np.testing.assert_array_equal(out, out_o)


@pytest.mark.parametrize("K", [1, 7, 2560, 6912])
def test_absmax_bit_exact(cuda_backend, K):
    rng = np.random.default_rng(K)
    x = (rng.standard_normal(K) * 10).astype(np.float32)
    x[0] = 0.5  # exercise ties
    qo = np.zeros(K, dtype=np.int8)
    import ctypes as C

    so = C.c_float()
    assert L.orc_absmax_quantize_row_into(p(x), K, p(qo), K, C.byref(so)) == 0
    q = np.zeros(K, dtype=np.int8)
    s = cuda_backend.absmax_quantize_row_into(x, q)
    np.testing.assert_array_equal(q, qo)
    assert np.float32(s) == np.float32(so.value)


@pytest.mark.parametrize("d", [1, 8, 13, 2560, 6912])
def test_rms_norm_bit_exact(cuda_backend, d):
    rng = np.random.default_rng(d)
    x = rng.standard_normal(d).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    oo = np.zeros(d, dtype=np.float32)
    assert L.orc_rms_norm(p(x), d, p(w), d, 1e-5, p(oo), d) == 0
    o = np.zeros(d, dtype=np.float32)
    cuda_backend.rms_norm(x, w, 1e-5, o)
    np.testing.assert_array_equal(o, oo)


@pytest.mark.parametrize("pos", [0, 1, 17, 4095, 5000])
def test_rope_bit_exact(cuda_backend, pos):
    rng = np.random.default_rng(pos)
    hd, nh, nkv = 128, 20, 5
    q = rng.standard_normal(nh * hd).astype(np.float32)
    k = rng.standard_normal(nkv * hd).astype(np.float32)
    qo, ko = q.copy(), k.copy()
    assert L.orc_rope_embed(p(qo), qo.size, p(ko), ko.size, pos, hd, nh, nkv, 500000.0) == 0
    cuda_backend.rope_embed(q, k, pos, hd, nh, nkv, 500000.0)
    np.testing.assert_array_equal(q, qo)
    np.testing.assert_array_equal(k, ko)


@pytest.mark.parametrize("seq_len,nh,nkv,hd", [(1, 20, 5, 128), (37, 20, 5, 128), (300, 4, 2, 12), (5, 2, 1, 4)])
def test_masked_attention_bit_exact(cuda_backend, seq_len, nh, nkv, hd):
    rng = np.random.default_rng(seq_len * 31 + hd)
    max_seq = seq_len + 3
    q = rng.standard_normal(nh * hd).astype(np.float32)
    kc = rng.standard_normal(nkv * max_seq * hd).astype(np.float32)
    vc = rng.standard_normal(nkv * max_seq * hd).astype(np.float32)
    oo = np.zeros(nh * hd, dtype=np.float32)
    assert L.orc_masked_attention(p(q), q.size, p(kc), kc.size, p(vc), vc.size, p(oo), oo.size, nh, nkv, hd,
                                  seq_len - 1) == 0
    o = np.zeros(nh * hd, dtype=np.float32)
    cuda_backend.masked_attention(q, kc, vc, o, nh, nkv, hd, seq_len - 1)
    np.testing.assert_array_equal(o, oo)


def test_elementwise_bit_exact(cuda_backend):
    rng = np.random.default_rng(0)
    n = 6912
    g = rng.standard_normal(n).astype(np.float32)
    u = rng.standard_normal(n).astype(np.float32)
    oo = np.zeros(n, dtype=np.float32)
    assert L.orc_sqrelu_gate(p(g), n, p(u), n, p(oo), n) == 0
    o = np.zeros(n, dtype=np.float32)
    cuda_backend.sqrelu_gate(g, u, o)
    np.testing.assert_array_equal(o, oo)
    x = g.copy()
    xo = g.copy()
    L.orc_squared_relu(p(xo), n)
    cuda_backend.squared_relu(x)
    np.testing.assert_array_equal(x, xo)
    L.orc_elementwise_mul(p(g), n, p(u), n, p(oo), n)
    cuda_backend.elementwise_mul(g, u, o)
    np.testing.assert_array_equal(o, oo)
    with pytest.raises(InvalidShape):
        cuda_backend.sqrelu_gate(g, u[:-1], o)


def test_softmax_exp_matches_host_libm_on_hard_inputs(cuda_backend):
    """Inputs where the host libm's expf is not the correctly rounded exp:
    the CUDA softmax still reproduces the reference (f32::exp -> libm expf)
    bit for bit."""
    import ctypes

    libm = ctypes.CDLL("libm.so.6")
    libm.expf.restype = ctypes.c_float
    libm.expf.argtypes = [ctypes.c_float]
    u = np.arange(0xBF000000, 0xBF000000 + 300000, dtype=np.uint32)  # x in (-0.5, -0.49]: ~1 in 1100 differ
    x = u.view(np.float32)
    cr = np.exp(x.astype(np.float64)).astype(np.float32)
    g = np.array([libm.expf(float(v)) for v in x], dtype=np.float32)
    hard = x[g != cr]
    assert hard.size >= 8, hard.size
    v = np.concatenate([[0.0], hard[:1024]]).astype(np.float32)  # max is 0, so exp(x - max) == exp(x)
    ref = v.copy()
    L.orc_softmax(p(ref), ref.size)
    got = v.copy()
    cuda_backend.softmax(got)
    np.testing.assert_array_equal(got, ref)


def test_softmax_bit_exact(cuda_backend):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(5000) * 4).astype(np.float32)
    xo = x.copy()
    L.orc_softmax(p(xo), xo.size)
    cuda_backend.softmax(x)
    np.testing.assert_array_equal(x, xo)


@pytest.mark.parametrize("V,H", [(1000, 2560), (37, 13), (300, 8)])
def test_lm_heads_bit_exact(cuda_backend, V, H):
    rng = np.random.default_rng(V + H)
    h = rng.standard_normal(H).astype(np.float32)
    w8 = rng.integers(-128, 128, size=V * H, dtype=np.int8)
    sc = (rng.random(V) * 0.01).astype(np.float32)
    oo = np.zeros(V, dtype=np.float32)
    o = np.zeros(V, dtype=np.float32)
    L.orc_lm_head_i8(p(h), p(w8), p(sc), p(oo), V, H)
    cuda_backend.lm_head_matmul_i8_into(h, w8, sc, o, V, H)
    np.testing.assert_array_equal(o, oo)
    wb = rng.integers(0, 65536, size=V * H, dtype=np.uint16)
    wb = np.where((wb & 0x7F80) == 0x7F80, wb & 0xBFFF, wb).astype(np.uint16)  # no inf/nan patterns
    L.orc_lm_head_bf16(p(h), p(wb), p(oo), V, H)
    cuda_backend.lm_head_matmul_bf16_into(h, wb, o, V, H)
    np.testing.assert_array_equal(o, oo)
    wf = rng.standard_normal(V * H).astype(np.float32)
    L.orc_lm_head_f32(p(h), p(wf), p(oo), V, H)
    cuda_backend.lm_head_matmul_into(h, wf, o, V, H)
    np.testing.assert_array_equal(o, oo)


@pytest.mark.parametrize("n", [1, 5, 1000, 128256])
def test_argmax_random(cuda_backend, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    if n > 10:
        x[n // 3] = x[2 * n // 3] = x.max() + 1  # tie -> later index
    assert cuda_backend.greedy_argmax(x) == L.orc_greedy_argmax(p(x), n)


def test_kernels_loaded_for_sm100(cuda_backend):
    """The driver loads the library's kernels as sm_100 SASS (the build embeds
    sm_100a only, so there is no PTX to fall back to)."""
    import ctypes as C

    from bitnetrs_b200 import _native as N

    v = C.c_int32(0)
    N.check(N.cuda_lib().bitnet_cuda_kernel_binary_version(C.byref(v)))
    assert v.value == 100, v.value
