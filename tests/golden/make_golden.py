"""Write tests/golden/kats.json: known-answer vectors of the bitnetrs hot path.

Every vector is transcribed from an assertion in the reference's own unit
tests (path:line given in "source"), or — for the tiny-model logits — computed
with the reference's analytic formula (crates/bitnet-model/src/lib.rs:1287-1319)
in float32 with the same left-to-right summation.  The reference is Rust and
cannot be built or run in this image, so these transcriptions are what pins
the CPU oracle (tests/test_oracle_kats.py) and, through it, the CUDA kernels.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

OUT = Path(__file__).with_name("kats.json")
f32 = np.float32


def bf16_round(x: float) -> float:
    u = np.array([x], dtype=np.float32).view(np.uint32).astype(np.uint64)[0]
    u = int(((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16) & 0xFFFFFFFF
    return float(np.array([u], dtype=np.uint32).view(np.float32)[0])


def analytical_logits_tiny(token_id: int):
    """model/src/lib.rs:1287-1319 (vocab 16, hidden 8, eps 1e-5)."""
    v, h, eps = 16, 8, f32(1e-5)
    center = f32(v * h // 2) * f32(0.01)
    embed = [f32(bf16_round(float(f32(token_id * h + i) * f32(0.01) - center))) for i in range(h)]
    sum_sq = f32(0.0)
    for x in embed:
        sum_sq = f32(sum_sq + f32(x * x))
    rms = f32(np.sqrt(f32(sum_sq / f32(h) + eps)))
    inv = f32(f32(1.0) / rms)
    out = []
    for vi in range(v):
        acc = f32(0.0)
        for hi in range(h):
            lm = f32(bf16_round(float(f32(vi * h + hi) * f32(0.01) - center)))
            acc = f32(acc + f32(f32(lm * embed[hi]) * inv))
        out.append(float(acc))
    return out


def round_half_away(y) -> float:
    """Rust f32::round (C roundf): halfway cases away from zero."""
    y = float(y)
    return float(np.sign(y) * np.floor(abs(y) + 0.5))


def hsum8(a):
    """hsum_f32_avx2 (crates/bitnet-cpu/src/simd.rs:292-307) on eight f32 lanes."""
    s = [f32(a[j] + a[j + 4]) for j in range(4)]
    return f32(f32(s[0] + s[1]) + f32(s[2] + s[3]))


def i8_head_logits_tiny(token_id: int):
    """The tiny model's logits through the i8 lm_head the forward pass actually
    uses (model/src/lib.rs:848 lm_head_matmul_i8_into; table of
    weights/src/loader.rs:297-340), in the AVX2 order of norm.rs:113-137 and
    simd.rs:1213-1250 (hidden size 8 = one 8-lane chunk, no scalar tail)."""
    v, h, eps = 16, 8, f32(1e-5)
    center = f32(v * h // 2) * f32(0.01)
    emb = lambda r: [f32(bf16_round(float(f32(r * h + i) * f32(0.01) - center))) for i in range(h)]  # noqa: E731
    x = emb(token_id)
    ss = hsum8([f32(t * t) for t in x])  # fma(x, x, 0) == round(x*x)
    inv = f32(f32(1.0) / f32(np.sqrt(f32(f32(ss / f32(h)) + eps))))
    hn = [f32(f32(t * inv) * f32(1.0)) for t in x]
    out = []
    for vi in range(v):
        row = emb(vi)
        m = max(abs(t) for t in row)
        m = max(m, f32(1e-10))
        inv_max = f32(f32(127.0) / m)
        scale = f32(m / f32(127.0))
        q = [f32(min(max(round_half_away(f32(t * inv_max)), -128.0), 127.0)) for t in row]
        out.append(float(f32(hsum8([f32(q[i] * hn[i]) for i in range(h)]) * scale)))
    return out


def kats():
    k = []

    def add(name, source, **kw):
        k.append(dict(name=name, source=source, **kw))

    # ---- pack_ternary / unpack_ternary (crates/bitnet-core/src/quant/ternary.rs) ----
    add("pack_spec", "crates/bitnet-core/src/quant/ternary.rs:361-375", fn="pack", values=[1, 0, -1, 1],
        packed=[0x24])
    add("pack_plus_ones", "crates/bitnet-core/src/quant/ternary.rs:385-393", fn="pack", values=[1, 1, 1, 1],
        packed=[0x00])
    add("pack_zeros", "crates/bitnet-core/src/quant/ternary.rs:395-397", fn="pack", values=[0, 0, 0, 0],
        packed=[0x55])
    add("pack_zero_row16", "crates/bitnet-core/src/quant/ternary.rs:400-410", fn="pack", values=[0] * 16,
        packed=[0x55] * 4)
    add("pack_neg_row16", "crates/bitnet-core/src/quant/ternary.rs:426-437", fn="pack", values=[-1] * 16,
        packed=[0xAA] * 4)
    add("pack_roundtrip_8", "crates/bitnet-core/src/quant/ternary.rs:343-349", fn="pack",
        values=[1, 0, -1, 1, -1, -1, 0, 0], packed_len=2, roundtrip=True)
    add("pack_roundtrip_3", "crates/bitnet-core/src/quant/ternary.rs:352-358", fn="pack", values=[1, -1, 0],
        packed_len=1, roundtrip=True)
    add("unpack_insufficient", "crates/bitnet-core/src/quant/ternary.rs:440-444", fn="unpack", packed=[0], n=8,
        error="InvalidShape")
    add("unpack_code_11", "crates/bitnet-core/src/quant/ternary.rs:309-316", fn="unpack", packed=[0xFF], n=4,
        error="QuantizationError")
    add("packed_bytes_rowaligned", "crates/bitnet-core/src/quant/ternary.rs:531-538", fn="packed_bytes",
        cases=[[4, 4, 4], [4, 5, 8], [3, 3, 3]])

    # ---- decode_packed_projection (crates/bitnet-convert/src/lib.rs) ----
    # lane at bits 2s of byte (r, c) -> logical row s*packed_rows + r, value lane-1
    add("hf_decode_expands_rows_by_four", "crates/bitnet-convert/src/lib.rs:821-853", fn="hf_decode",
        packed=[0b01_10_01_00] * 8, packed_rows=2, cols=4, scale=2.0,
        rows=[[-1] * 4, [-1] * 4, [0] * 4, [0] * 4, [1] * 4, [1] * 4, [0] * 4, [0] * 4])
    # the documented error conditions (lib.rs:228-233) in the order of the checks (lib.rs:243-290)
    add("hf_decode_zero_rows", "crates/bitnet-convert/src/lib.rs:243-245", fn="hf_decode", packed=[0] * 4,
        packed_rows=0, cols=4, scale=1.0, error="InvalidShape")
    add("hf_decode_zero_cols", "crates/bitnet-convert/src/lib.rs:246-248", fn="hf_decode", packed=[0] * 4,
        packed_rows=1, cols=0, scale=1.0, error="InvalidShape")
    add("hf_decode_bad_scale", "crates/bitnet-convert/src/lib.rs:249-253", fn="hf_decode", packed=[0x55] * 4,
        packed_rows=1, cols=4, scale=0.0, error="QuantizationError")
    add("hf_decode_short", "crates/bitnet-convert/src/lib.rs:262-270", fn="hf_decode", packed=[0x55] * 3,
        packed_rows=1, cols=4, scale=1.0, error="InvalidShape")
    add("hf_decode_lane_11", "crates/bitnet-convert/src/lib.rs:279-283", fn="hf_decode",
        packed=[0x55, 0x55, 0x55, 0x55, 0x55, 0x55, 0x55, 0b00_11_01_01], packed_rows=2, cols=4, scale=1.0,
        error="QuantizationError", message="(1, 3), shift 4")

    # ---- sample_next_token (crates/bitnet-inference/src/lib.rs:236-390) ----
    def cfg(temperature=1.0, top_p=1.0, top_k=0, repetition_penalty=1.0, seed=0):
        return dict(temperature=temperature, top_p=top_p, top_k=top_k, repetition_penalty=repetition_penalty,
                    seed=seed)

    greedy = cfg(top_k=1, seed=42)  # SamplingConfig::greedy (lib.rs:115-124)
    add("sample_greedy_argmax", "crates/bitnet-inference/src/lib.rs:1094-1101", fn="sample",
        logits=[0.1, 0.5, 5.0, 0.2, -1.0], cfg=greedy, past=[], token=2)
    add("sample_greedy_last_max", "crates/bitnet-inference/src/lib.rs:1104-1110", fn="sample",
        logits=[0.0, 0.0, 0.0, 0.0, 10.0], cfg=greedy, past=[], token=4)
    add("sample_greedy_first_max", "crates/bitnet-inference/src/lib.rs:1113-1119", fn="sample",
        logits=[100.0, 0.0, -1.0, -5.0], cfg=greedy, past=[], token=0)
    add("sample_only_finite_token", "crates/bitnet-inference/src/lib.rs:1226-1243", fn="sample",
        logits=["-inf"] * 5 + [1.0] + ["-inf"] * 2, cfg=cfg(), past=[], token=5)
    add("sample_top_k_1", "crates/bitnet-inference/src/lib.rs:1246-1263", fn="sample",
        logits=[1.0, 5.0, 0.0, -1.0, 2.0], cfg=cfg(top_k=1), past=[], token=1)
    add("sample_low_temperature", "crates/bitnet-inference/src/lib.rs:1266-1283", fn="sample",
        logits=[0.0, 1.0, 10.0, 2.0], cfg=cfg(temperature=0.01), past=[], token=2)
    add("sample_top_k_3_over_seeds", "crates/bitnet-inference/src/lib.rs:1958-1983", fn="sample",
        logits=[1.0, 5.0, 3.0, 2.0, 4.0, 0.5], cfg=cfg(temperature=2.0, top_k=3), past=[], seeds=50,
        allowed=[1, 4, 2])
    add("sample_in_range", "crates/bitnet-inference/src/lib.rs:1122-1140", fn="sample",
        logits=[float(f32(i) * f32(0.1)) for i in range(32)], cfg=cfg(temperature=0.8, top_p=0.9, top_k=10, seed=42),
        past=[], allowed=list(range(32)))
    add("sample_repetition_penalty", "crates/bitnet-inference/src/lib.rs:1143-1169", fn="sample",
        logits=[0.0, 0.0, 10.0, 0.0], cfg=cfg(repetition_penalty=1000.0, seed=42), past=[2], allowed=[0, 1, 2, 3])
    # SamplingConfig::validate (lib.rs:160-178) on the presets and the rejected variants (lib.rs:1024-1090)
    add("sampling_config_presets", "crates/bitnet-inference/src/lib.rs:1024-1090", fn="sampling_config",
        valid=["greedy", "chat_defaults", "creative", "default"],
        invalid=[{"temperature": 0.0}, {"top_p": 1.5}, {"top_p": 0.0}, {"repetition_penalty": 0.9},
                 {"max_new_tokens": 0}])

    # ---- absmax_quantize_row (crates/bitnet-core/src/quant/absmax.rs) ----
    add("absmax_max_is_127", "crates/bitnet-core/src/quant/absmax.rs:291-300", fn="absmax", x=[0.0, 1.0, 2.0, -1.0],
        q_at={"2": 127, "3": -64}, scale=2.0 / 127.0, scale_tol=1e-7)
    add("absmax_neg_max", "crates/bitnet-core/src/quant/absmax.rs:303-313", fn="absmax", x=[-3.0, 0.0, 1.5],
        q=[-127, 0, 64], scale=3.0 / 127.0, scale_tol=1e-7)
    add("absmax_zeros", "crates/bitnet-core/src/quant/absmax.rs:316-321", fn="absmax", x=[0.0] * 8, q=[0] * 8,
        scale_positive=True)
    add("absmax_empty", "crates/bitnet-core/src/quant/absmax.rs:324-327", fn="absmax", x=[],
        error="QuantizationError")
    add("absmax_nan", "crates/bitnet-core/src/quant/absmax.rs:330-333", fn="absmax", x=[1.0, "nan"],
        error="QuantizationError")
    add("absmax_inf", "crates/bitnet-core/src/quant/absmax.rs:336-339", fn="absmax", x=[1.0, "inf"],
        error="QuantizationError")
    add("absmax_single_pos", "crates/bitnet-core/src/quant/absmax.rs:368-373", fn="absmax", x=[5.0], q=[127],
        scale=5.0 / 127.0, scale_tol=1e-6)
    add("absmax_single_neg", "crates/bitnet-core/src/quant/absmax.rs:376-380", fn="absmax", x=[-4.0], q=[-127],
        scale=4.0 / 127.0, scale_tol=1e-6)
    add("absmax_doc", "crates/bitnet-core/src/quant/absmax.rs:69-75", fn="absmax", x=[0.0, 1.0, -2.0, 0.5],
        q_at={"2": -127})

    # ---- absmean_quantize (crates/bitnet-core/src/quant/absmean.rs) ----
    add("absmean_positive", "crates/bitnet-core/src/quant/absmean.rs:213-222", fn="absmean", w=[0.4, 0.8, 1.2, 0.0],
        q=[1, 1, 1, 0], scale=0.6, scale_tol=1e-5)
    add("absmean_mixed", "crates/bitnet-core/src/quant/absmean.rs:225-233", fn="absmean", w=[0.5, -0.5, 0.0, -1.5],
        q=[1, -1, 0, -1], scale=0.625, scale_tol=1e-5)
    add("absmean_zeros", "crates/bitnet-core/src/quant/absmean.rs:236-244", fn="absmean", w=[0.0] * 8, q=[0] * 8,
        scale=1e-5, scale_tol=0.0)
    add("absmean_single_pos", "crates/bitnet-core/src/quant/absmean.rs:290-296", fn="absmean", w=[2.5], q=[1],
        scale=2.5, scale_tol=1e-6)
    add("absmean_single_neg", "crates/bitnet-core/src/quant/absmean.rs:299-303", fn="absmean", w=[-3.0], q=[-1],
        scale=3.0, scale_tol=1e-6)
    add("absmean_doc", "crates/bitnet-core/src/quant/absmean.rs:62-70", fn="absmean", w=[0.3, -0.6, 0.0, 1.2],
        q=[1, -1, 0, 1])
    add("absmean_pm1", "crates/bitnet-cpu/src/gemv.rs:566-582", fn="absmean",
        w=[1.0, -1.0, 1.0, -1.0, 1.0, 1.0, -1.0, -1.0], q=[1, -1, 1, -1, 1, 1, -1, -1], scale=1.0, scale_tol=1e-5)
    add("absmean_empty", "crates/bitnet-core/src/quant/absmean.rs:247-253", fn="absmean", w=[],
        error="QuantizationError")
    add("absmean_nan", "crates/bitnet-core/src/quant/absmean.rs:256-259", fn="absmean", w=[1.0, "nan", 0.0],
        error="QuantizationError")

    # ---- ternary GEMV f32 path (crates/bitnet-cpu/src/gemv.rs) ----
    add("gemv_2x3", "crates/bitnet-cpu/src/gemv.rs:419-430", fn="gemv_f32", w=[[1, 0, -1], [-1, 1, 0]], scale=0.5,
        x=[2.0, 3.0, 4.0], out=[-1.0, 0.5], tol=1e-6)
    add("gemv_identity", "crates/bitnet-cpu/src/gemv.rs:433-444", fn="gemv_f32",
        w=[[1, 0, 0], [0, 1, 0], [0, 0, 1]], scale=1.0, x=[5.0, 7.0, 9.0], out=[5.0, 7.0, 9.0], tol=1e-6)
    add("gemv_negation", "crates/bitnet-cpu/src/gemv.rs:447-457", fn="gemv_f32", w=[[-1, -1, -1, -1]], scale=2.0,
        x=[1.0, 2.0, 3.0, 4.0], out=[-20.0], tol=1e-5)
    add("gemv_scale", "crates/bitnet-cpu/src/gemv.rs:460-469", fn="gemv_f32", w=[[1, 1, 1]], scale=0.25,
        x=[1.0, 1.0, 1.0], out=[0.75], tol=1e-7)
    add("gemv_1x1", "crates/bitnet-cpu/src/gemv.rs:535-544", fn="gemv_f32", w=[[-1]], scale=2.0, x=[3.0], out=[-6.0],
        tol=1e-7)
    add("gemv_zero_w", "crates/bitnet-cpu/src/gemv.rs:547-559", fn="gemv_f32", w=[[0] * 4] * 3, scale=1.0,
        x=[99.0] * 4, out=[0.0] * 3, tol=0.0)
    add("gemv_bad_weight_len", "crates/bitnet-cpu/src/gemv.rs:471-481", fn="gemv_f32_raw", packed_len=3, N=2, K=3,
        x_len=3, out_len=2, scale=1.0, error="InvalidShape")
    add("gemv_bad_input_len", "crates/bitnet-cpu/src/gemv.rs:484-494", fn="gemv_f32_raw", packed_len=2, N=2, K=3,
        x_len=4, out_len=2, scale=1.0, error="InvalidShape")
    add("gemv_bad_output_len", "crates/bitnet-cpu/src/gemv.rs:497-507", fn="gemv_f32_raw", packed_len=2, N=2, K=3,
        x_len=3, out_len=3, scale=1.0, error="InvalidShape")
    add("gemv_zero_scale", "crates/bitnet-cpu/src/gemv.rs:510-520", fn="gemv_f32_raw", packed_len=1, N=1, K=4,
        x_len=4, out_len=1, scale=0.0, error="QuantizationError")
    add("gemv_neg_scale", "crates/bitnet-cpu/src/gemv.rs:523-532", fn="gemv_f32_raw", packed_len=1, N=1, K=4,
        x_len=4, out_len=1, scale=-0.5, error="QuantizationError")

    # ---- integer dot products (gemv.rs tests, simd.rs AVX2 edge cases) ----
    add("dot_i8_basic", "crates/bitnet-cpu/src/gemv.rs:376-381", fn="dot_i8", w=[1, -1, 0], x=[100, 50, 127], acc=50)
    add("dot_i8_508", "crates/bitnet-cpu/src/gemv.rs:384-389", fn="dot_i8", w=[1] * 4, x=[127] * 4, acc=508)
    add("dot_i8_cancel", "crates/bitnet-cpu/src/gemv.rs:392-398", fn="dot_i8", w=[1, 1, -1, -1], x=[64] * 4, acc=0)
    add("dot_i8_127x64", "crates/bitnet-cpu/src/simd.rs:1556-1566", fn="dot_i8", w=[1] * 64, x=[127] * 64,
        acc=64 * 127)
    add("dot_i8_neg128_pos", "crates/bitnet-cpu/src/simd.rs:1568-1577", fn="dot_i8", w=[1] * 64, x=[-128] * 64,
        acc=-8192)
    add("dot_i8_neg128_neg", "crates/bitnet-cpu/src/simd.rs:1579-1590", fn="dot_i8", w=[-1] * 64, x=[-128] * 64,
        acc=8192)

    # ---- quantised GEMV formula (gemv.rs:563-674) ----
    add("gemv_q_consistent", "crates/bitnet-cpu/src/gemv.rs:563-627", fn="gemv_q_formula",
        w=[1.0, -1.0, 1.0, -1.0, 1.0, 1.0, -1.0, -1.0], rows=2, cols=4, x=[2.0, 2.0, 2.0, 2.0], tol=1e-6, expect="acc*ws*x_scale/127")
    add("gemv_q_nonzero", "crates/bitnet-cpu/src/gemv.rs:630-658", fn="gemv_q_formula", w=[1.0, 1.0, 1.0, 1.0],
        rows=1, cols=4, x=[1.0, 0.0, 0.0, 0.0], tol=1e-6, expect="acc*ws*max_abs/127")
    add("gemv_q_bad_act_scale", "crates/bitnet-cpu/src/gemv.rs:661-671", fn="gemv_q_raw", w=[[1, 1, 1, 1]],
        scale=1.0, xq=[100] * 4, act_absmax=0.0, error="QuantizationError")

    # ---- RMSNorm (crates/bitnet-cpu/src/norm.rs) ----
    add("rms_norm_doc", "crates/bitnet-cpu/src/norm.rs:66-75", fn="rms_norm", x=[1.0, 2.0, 3.0, 4.0], w=[1.0] * 4,
        eps=1e-5, out_at={"0": float(f32(1.0) / np.sqrt(f32(7.5) + f32(1e-5)))}, tol=1e-5)
    add("rms_norm_zero", "crates/bitnet-cpu/src/norm.rs:246-256", fn="rms_norm", x=[0.0] * 8, w=[1.0] * 8, eps=1e-5,
        out=[0.0] * 8, tol=0.0)
    add("rms_norm_len_mismatch", "crates/bitnet-cpu/src/norm.rs:77-91", fn="rms_norm", x=[1.0, 2.0], w=[1.0],
        eps=1e-5, error="InvalidShape")
    add("rms_norm_bad_eps", "crates/bitnet-cpu/src/norm.rs:92-96", fn="rms_norm", x=[1.0], w=[1.0], eps=0.0,
        error="QuantizationError")

    # ---- RoPE (crates/bitnet-cpu/src/rope.rs) ----
    c1, s1 = float(np.cos(f32(1.0))), float(np.sin(f32(1.0)))
    add("rope_pos0_identity", "crates/bitnet-cpu/src/lib.rs:715-731", fn="rope", q=[1.0, 0.5, -0.3, 0.8],
        k=[0.1, -0.6, 0.4, -0.2], pos=0, head_dim=4, n_heads=1, n_kv_heads=1, theta=10000.0,
        q_out=[1.0, 0.5, -0.3, 0.8], k_out=[0.1, -0.6, 0.4, -0.2], tol=1e-6)
    add("rope_90deg", "crates/bitnet-cpu/src/rope.rs:648-677", fn="rope", q=[1.0, 0.0], k=[1.0, 0.0], pos=1,
        head_dim=2, n_heads=1, n_kv_heads=1, theta=10000.0, q_out=[c1, s1], k_out=[c1, s1], tol=1e-5)
    add("rope_odd_head_dim", "crates/bitnet-cpu/src/rope.rs:626-634", fn="rope", q=[0.0] * 3, k=[0.0] * 3, pos=0,
        head_dim=3, n_heads=1, n_kv_heads=1, theta=10000.0, error="InvalidConfig")
    add("rope_zero_theta", "crates/bitnet-cpu/src/rope.rs:637-645", fn="rope", q=[0.0] * 8, k=[0.0] * 8, pos=0,
        head_dim=8, n_heads=1, n_kv_heads=1, theta=0.0, error="InvalidConfig")
    add("rope_bad_q_len", "crates/bitnet-cpu/src/rope.rs:604-612", fn="rope", q=[0.0] * 7, k=[0.0] * 8, pos=0,
        head_dim=8, n_heads=1, n_kv_heads=1, theta=10000.0, error="InvalidShape")

    # ---- attention (crates/bitnet-cpu/src/attention.rs) ----
    add("attn_single_pos", "crates/bitnet-cpu/src/attention.rs:249-268", fn="attention", q=[1.0, 0.0, 0.0, 0.0],
        k=[1.0, 0.0, 0.0, 0.0], v=[0.1, 0.2, 0.3, 0.4], n_heads=1, n_kv_heads=1, head_dim=4, cur_pos=0,
        out=[0.1, 0.2, 0.3, 0.4], tol=1e-5)
    add("attn_uniform", "crates/bitnet-cpu/src/attention.rs:271-311", fn="attention", q=[0.0, 0.0],
        k=[1.0, 2.0, 3.0, 4.0, 5.0, 6.0], v=[1.0, 0.0, 2.0, 0.0, 3.0, 0.0], n_heads=1, n_kv_heads=1, head_dim=2,
        cur_pos=2, out=[2.0, 0.0], tol=1e-5)
    add("attn_gqa_indivisible", "crates/bitnet-cpu/src/attention.rs:118-122", fn="attention", q=[0.0] * 6,
        k=[0.0] * 4, v=[0.0] * 4, n_heads=3, n_kv_heads=2, head_dim=2, cur_pos=0, error="InvalidConfig")

    # ---- greedy sampling (crates/bitnet-inference/src/lib.rs) ----
    add("argmax_basic", "crates/bitnet-inference/src/lib.rs:1094-1101", fn="argmax",
        logits=[0.1, 0.5, 5.0, 0.2, -1.0], token=2)
    add("argmax_last", "crates/bitnet-inference/src/lib.rs:1104-1110", fn="argmax", logits=[0.0, 0.0, 0.0, 0.0, 10.0],
        token=4)
    add("argmax_first", "crates/bitnet-inference/src/lib.rs:1113-1119", fn="argmax", logits=[100.0, 0.0, -1.0, -5.0],
        token=0)
    # Iterator::max_by returns the last of equal maxima (inference/lib.rs:263-274).
    add("argmax_tie_last", "crates/bitnet-inference/src/lib.rs:263-274", fn="argmax", logits=[3.0, 1.0, 3.0, 2.0],
        token=2)
    # partial_cmp(NaN) -> Equal: the fold restarts after the last NaN.
    add("argmax_nan_restart", "crates/bitnet-inference/src/lib.rs:263-274", fn="argmax",
        logits=[9.0, "nan", 1.0, 2.0], token=3)
    add("argmax_nan_last", "crates/bitnet-inference/src/lib.rs:263-274", fn="argmax", logits=[9.0, 1.0, "nan"],
        token=2)

    # ---- tiny model golden logits (crates/bitnet-model/src/lib.rs:1589-1646) ----
    # The reference asserts 1e-4 against a formula with a bf16 lm_head
    # (model/src/lib.rs:1287-1319), but its forward pass uses the i8 lm_head
    # (lib.rs:848), whose quantisation error on this model reaches ~4e-3; the
    # formula is therefore pinned at 5e-3, and the i8-head recomputation in
    # the reference's exact operation order at 1e-6.
    add("tiny_single_token", "crates/bitnet-model/src/lib.rs:1589-1617", fn="tiny_model", tokens=[0],
        logits=analytical_logits_tiny(0), tol=5e-3)
    add("tiny_prefill_2", "crates/bitnet-model/src/lib.rs:1620-1646", fn="tiny_model", tokens=[3, 7],
        logits=analytical_logits_tiny(7), tol=5e-3)
    add("tiny_single_token_i8_head", "crates/bitnet-model/src/lib.rs:848; crates/bitnet-weights/src/loader.rs:297-340",
        fn="tiny_model", tokens=[0], logits=i8_head_logits_tiny(0), tol=1e-6)
    add("tiny_prefill_2_i8_head", "crates/bitnet-model/src/lib.rs:848; crates/bitnet-weights/src/loader.rs:297-340",
        fn="tiny_model", tokens=[3, 7], logits=i8_head_logits_tiny(7), tol=1e-6)
    return k


if __name__ == "__main__":
    OUT.write_text(json.dumps({"generator": "tests/golden/make_golden.py", "kats": kats()}, indent=1) + "\n")
    print(OUT)
