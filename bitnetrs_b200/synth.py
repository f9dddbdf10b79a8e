"""Seeded synthetic models and inputs (no checkpoint exists on the benchmark boxes).

Random-init weights go through the reference's own quantisation pipeline
(absmean ternarisation + 2-bit packing for projections, bf16 embedding with a
weight-tied per-row absmax i8 lm_head), see ``csrc/synth.cpp``.

Stream ids: embedding 1; layer ``l`` tensor ``j`` (q,k,v,o,gate,up,down =
0..6) uses ``1000 + 16*l + j``.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from .model import LayerWeights, ModelConfig, ModelWeights


def set_threads(n: int) -> int:
    return N.synth_lib().synth_set_threads(n)


def normal_f32(seed: int, stream: int, n: int, std: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    N.synth_lib().synth_normal_f32(seed, stream, offset, n, std, out.ctypes.data)
    return out


def bf16_normal(seed: int, stream: int, n: int, std: float) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    N.synth_lib().synth_bf16_normal(seed, stream, n, std, out.ctypes.data)
    return out


def ternary_absmean(seed: int, stream: int, rows: int, cols: int, std: float):
    """N(0,std) weights -> absmean ternary -> reference packed rows; returns (packed uint8, scale)."""
    out = np.empty(rows * ((cols + 3) // 4), dtype=np.uint8)
    s = C.c_float()
    rc = N.synth_lib().synth_ternary_absmean(seed, stream, rows, cols, std, out.ctypes.data, C.byref(s))
    if rc:
        raise ValueError("empty tensor")
    return out, s.value


def ternary_codes(seed: int, stream: int, rows: int, cols: int, p_neg: float = 0.34, p_zero: float = 0.32):
    """iid ternary weights with P(-1)=p_neg, P(0)=p_zero, packed in the reference format."""
    out = np.empty(rows * ((cols + 3) // 4), dtype=np.uint8)
    N.synth_lib().synth_ternary_codes(seed, stream, rows, cols, p_neg, p_zero, out.ctypes.data)
    return out


def quantize_bf16_rows_to_i8(embed_bf16: np.ndarray, rows: int, row_len: int):
    """loader.rs:297-340: per-row absmax int8 table + scales for the tied lm_head."""
    q = np.empty(rows * row_len, dtype=np.int8)
    s = np.empty(rows, dtype=np.float32)
    N.synth_lib().synth_quantize_bf16_rows_to_i8(embed_bf16.ctypes.data, rows, row_len, q.ctypes.data, s.ctypes.data)
    return q, s


def uniform_u32(seed: int, stream: int, n: int, lo: int, hi: int) -> np.ndarray:
    out = np.empty(n, dtype=np.uint32)
    N.synth_lib().synth_uniform_u32(seed, stream, n, lo, hi, out.ctypes.data)
    return out


def kv_normal(seed: int, seq: int, cfg: ModelConfig, n: int):
    """Host copy of what ``KVCache.fill_random(seq, n, seed)`` writes (before bf16 rounding)."""
    L, nkv, hd = cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim()
    k = np.empty((L, n, nkv * hd), dtype=np.float32)
    v = np.empty_like(k)
    N.synth_lib().synth_kv_normal(seed, seq, L, nkv, hd, n, k.ctypes.data, v.ctypes.data)
    return k, v


def random_model(cfg: ModelConfig, seed: int = 0, std: float = 0.02, norm_gain: float = 1.0) -> ModelWeights:
    """Random-init model with the reference's weight formats (weights N(0, 0.02), norm gains 1.0)."""
    H, F, V, qd, kvd = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.q_dim(), cfg.kv_dim()
    layers = []
    for l in range(cfg.num_hidden_layers):
        base = 1000 + 16 * l
        q, sq = ternary_absmean(seed, base + 0, qd, H, std)
        k, sk = ternary_absmean(seed, base + 1, kvd, H, std)
        v, sv = ternary_absmean(seed, base + 2, kvd, H, std)
        o, so = ternary_absmean(seed, base + 3, H, qd, std)
        g, sg = ternary_absmean(seed, base + 4, F, H, std)
        u, su = ternary_absmean(seed, base + 5, F, H, std)
        d, sd = ternary_absmean(seed, base + 6, H, F, std)
        ones = lambda n: np.full(n, norm_gain, dtype=np.float32)  # noqa: E731
        layers.append(LayerWeights(q, k, v, o, g, u, d, sq, sk, sv, so, sg, su, sd, ones(H), ones(qd), ones(H),
                                   ones(F)))
    embed = bf16_normal(seed, 1, V * H, std)
    lm_i8, lm_s = quantize_bf16_rows_to_i8(embed, V, H)
    return ModelWeights(cfg, embed, lm_i8, lm_s, np.full(H, norm_gain, dtype=np.float32), layers)


# absmean ternarisation of N(0, s) weights zeroes |w| < 0.5 * E|w| = 0.5 *
# sqrt(2/pi) * s: P(0) = 2 * Phi(0.5 * sqrt(2/pi)) - 1, and the scale is E|w|.
ABSMEAN_P_ZERO = 0.3100643
ABSMEAN_SCALE_PER_STD = 0.7978846


def random_model_iid(cfg: ModelConfig, seed: int = 0, std: float = 0.02, norm_gain: float = 1.0) -> ModelWeights:
    """Random-init model whose ternary codes are drawn directly from the
    distribution absmean ternarisation of N(0, std) weights produces (P(0) =
    0.310, P(+1) = P(-1) = 0.345, per-tensor scale std * sqrt(2/pi)) instead
    of ternarising drawn weights: the same distributions and formats as
    :func:`random_model` at a fraction of the host time, for benchmark
    shapes whose exact values no test compares."""
    H, F, V, qd, kvd = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.q_dim(), cfg.kv_dim()
    p_pm = (1.0 - ABSMEAN_P_ZERO) / 2.0
    scale = float(np.float32(std * ABSMEAN_SCALE_PER_STD))
    layers = []
    for l in range(cfg.num_hidden_layers):
        base = 1000 + 16 * l
        shapes = [(qd, H), (kvd, H), (kvd, H), (H, qd), (F, H), (F, H), (H, F)]
        t = [ternary_codes(seed, base + j, r, c, p_pm, ABSMEAN_P_ZERO) for j, (r, c) in enumerate(shapes)]
        ones = lambda n: np.full(n, norm_gain, dtype=np.float32)  # noqa: E731
        layers.append(LayerWeights(*t, *([scale] * 7), ones(H), ones(qd), ones(H), ones(F)))
    embed = bf16_normal(seed, 1, V * H, std)
    lm_i8, lm_s = quantize_bf16_rows_to_i8(embed, V, H)
    return ModelWeights(cfg, embed, lm_i8, lm_s, np.full(H, norm_gain, dtype=np.float32), layers)


def tiny_reference_model(cfg: ModelConfig) -> ModelWeights:
    """The reference's golden tiny model (model/src/lib.rs:1459-1545): all-zero
    ternary projections (0x55 bytes, scale 1.0), unit norms, embedding
    bf16(i*0.01 - V*H/2*0.01), lm_head i8 table built from it."""
    H, F, V, qd, kvd = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.q_dim(), cfg.kv_dim()
    pc = lambda k: (k + 3) // 4  # noqa: E731
    zero = lambda r, c: np.full(r * pc(c), 0x55, dtype=np.uint8)  # noqa: E731
    ones = lambda n: np.ones(n, dtype=np.float32)  # noqa: E731
    layers = [LayerWeights(zero(qd, H), zero(kvd, H), zero(kvd, H), zero(H, qd), zero(F, H), zero(F, H), zero(H, F),
                           1.0, 1.0, 1.0, 1.0, 1.0, 1.0, 1.0, ones(H), ones(qd), ones(H), ones(F))
              for _ in range(cfg.num_hidden_layers)]
    vals = np.arange(V * H, dtype=np.float32) * np.float32(0.01) - np.float32(V * H // 2) * np.float32(0.01)
    embed = f32_to_bf16_bits(vals)
    lm_i8, lm_s = quantize_bf16_rows_to_i8(embed, V, H)
    return ModelWeights(cfg, embed, lm_i8, lm_s, ones(H), layers)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """half::bf16::from_f32 (round to nearest even) on a float32 array."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, ((u | 0x00400000) >> 16) & 0xFFFF, r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
