"""ctypes wrapper of the CPU oracle (oracle/liboracle.so) — test infrastructure.

The oracle restates the reference CPU backend; tests use it only as the
checker for the CUDA backend.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "oracle" / "liboracle.so"

vp, sz, f32, u32, i32 = C.c_void_p, C.c_size_t, C.c_float, C.c_uint32, C.c_int


class Cfg(C.Structure):
    _fields_ = [("vocab_size", u32), ("hidden_size", u32), ("num_layers", u32), ("num_heads", u32),
                ("num_kv_heads", u32), ("intermediate_size", u32), ("max_position", u32), ("rope_theta", f32),
                ("rms_norm_eps", f32)]


class Layer(C.Structure):
    _fields_ = [("q", vp), ("k", vp), ("v", vp), ("o", vp), ("gate", vp), ("up", vp), ("down", vp),
                ("sq", f32), ("sk", f32), ("sv", f32), ("so", f32), ("sg", f32), ("su", f32), ("sd", f32),
                ("attn_norm", vp), ("attn_sub_norm", vp), ("ffn_norm", vp), ("ffn_sub_norm", vp)]


class Weights(C.Structure):
    _fields_ = [("embed", vp), ("lm_head_i8", vp), ("lm_head_scales", vp), ("final_norm", vp),
                ("layers", C.POINTER(Layer))]


_SIGS = {
    "orc_set_threads": (i32, [i32]),
    "orc_threads": (i32, []),
    "orc_has_avx2_fma": (i32, []),
    "orc_pack_ternary": (None, [vp, sz, vp]),
    "orc_unpack_ternary": (i32, [vp, sz, sz, vp]),
    "orc_absmean_quantize": (i32, [vp, sz, vp, C.POINTER(f32)]),
    "orc_decode_hf_packed": (i32, [vp, sz, sz, sz, f32, vp]),
    "orc_sample_next_token": (C.c_uint32, [vp, sz, f32, f32, sz, f32, C.c_uint64, vp, sz]),
    "orc_absmax_quantize_row_into": (i32, [vp, sz, vp, sz, C.POINTER(f32)]),
    "orc_quantize_bf16_rows_to_i8": (None, [vp, sz, sz, vp, vp]),
    "orc_bf16_round": (f32, [f32]),
    "orc_ternary_gemv": (i32, [vp, sz, f32, vp, sz, vp, sz, sz, sz]),
    "orc_ternary_gemv_preq": (i32, [vp, sz, f32, vp, sz, f32, vp, sz, sz, sz, vp]),
    "orc_ternary_gemv_with_activation_quant": (i32, [vp, sz, f32, vp, sz, vp, sz, sz, sz]),
    "orc_rms_norm": (i32, [vp, sz, vp, sz, f32, vp, sz]),
    "orc_rope_embed": (i32, [vp, sz, vp, sz, sz, sz, sz, sz, f32]),
    "orc_masked_attention": (i32, [vp, sz, vp, sz, vp, sz, vp, sz, sz, sz, sz, sz]),
    "orc_squared_relu": (None, [vp, sz]),
    "orc_softmax": (None, [vp, sz]),
    "orc_elementwise_mul": (i32, [vp, sz, vp, sz, vp, sz]),
    "orc_sqrelu_gate": (i32, [vp, sz, vp, sz, vp, sz]),
    "orc_lm_head_f32": (i32, [vp, vp, vp, sz, sz]),
    "orc_lm_head_bf16": (i32, [vp, vp, vp, sz, sz]),
    "orc_lm_head_i8": (i32, [vp, vp, vp, vp, sz, sz]),
    "orc_greedy_argmax": (u32, [vp, sz]),
    "orc_model_create": (vp, [C.POINTER(Cfg), C.POINTER(Weights)]),
    "orc_model_destroy": (None, [vp]),
    "orc_kv_create": (vp, [vp, sz, i32]),
    "orc_kv_destroy": (None, [vp]),
    "orc_kv_clear": (None, [vp]),
    "orc_kv_len": (sz, [vp]),
    "orc_kv_seed": (i32, [vp, sz, vp, vp]),
    "orc_kv_read": (i32, [vp, sz, vp, vp]),
    "orc_forward": (i32, [vp, vp, vp, sz, sz, vp]),
    "orc_generate": (i32, [vp, vp, vp, sz, sz, u32, u32, vp, C.POINTER(sz), vp]),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            subprocess.run(["make", "-C", str(LIB.parent)], check=True, capture_output=True)
        L = C.CDLL(str(LIB))
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def p(a):
    return None if a is None else a.ctypes.data


ERR = {0: None, 1: "InvalidShape", 2: "QuantizationError", 3: "BackendError", 4: "InvalidConfig"}


class OracleModel:
    """The reference forward pass (BitNetModel::forward) on host weights."""

    def __init__(self, weights):
        c = weights.config
        self.config = c
        self._cfg = Cfg(c.vocab_size, c.hidden_size, c.num_hidden_layers, c.num_attention_heads,
                        c.num_key_value_heads, c.intermediate_size, c.max_position_embeddings, c.rope_theta,
                        c.rms_norm_eps)
        self._layers = (Layer * len(weights.layers))()
        for i, L in enumerate(weights.layers):
            self._layers[i] = Layer(p(L.q_proj), p(L.k_proj), p(L.v_proj), p(L.o_proj), p(L.gate_proj), p(L.up_proj),
                                    p(L.down_proj), L.q_scale, L.k_scale, L.v_scale, L.o_scale, L.gate_scale,
                                    L.up_scale, L.down_scale, p(L.attention_norm), p(L.attn_sub_norm), p(L.ffn_norm),
                                    p(L.ffn_sub_norm))
        self._w = Weights(p(weights.embed_tokens), p(weights.lm_head_i8), p(weights.lm_head_scales),
                          p(weights.final_norm), self._layers)
        self._keep = weights
        self._h = lib().orc_model_create(C.byref(self._cfg), C.byref(self._w))

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_model_destroy(self._h)
            self._h = None

    def kv(self, max_seq, bf16=False):
        return OracleKV(self, max_seq, bf16)

    def forward(self, kv, tokens, start_pos):
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        out = np.empty(self.config.vocab_size, dtype=np.float32)
        rc = lib().orc_forward(self._h, kv._h, p(t), t.size, start_pos, p(out))
        if rc:
            raise RuntimeError(f"oracle forward failed: {ERR[rc]}")
        return out

    def generate(self, kv, prompt, max_new, eos=(128009, 128001)):
        pr = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        out = np.empty(max(1, max_new), dtype=np.uint32)
        margins = np.empty(max(1, max_new), dtype=np.float32)
        n = C.c_size_t()
        rc = lib().orc_generate(self._h, kv._h, p(pr), pr.size, max_new, eos[0], eos[1], p(out), C.byref(n),
                                p(margins))
        if rc:
            raise RuntimeError(f"oracle generate failed: {ERR[rc]}")
        return out[: n.value].tolist(), margins[: n.value]


class OracleKV:
    def __init__(self, model, max_seq, bf16=False):
        self._model = model
        self._h = lib().orc_kv_create(model._h, max_seq, 1 if bf16 else 0)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_kv_destroy(self._h)
            self._h = None

    def clear(self):
        lib().orc_kv_clear(self._h)

    def __len__(self):
        return lib().orc_kv_len(self._h)

    def read(self, n):
        c = self._model.config
        k = np.empty((c.num_hidden_layers, n, c.kv_dim()), dtype=np.float32)
        v = np.empty_like(k)
        rc = lib().orc_kv_read(self._h, n, p(k), p(v))
        if rc:
            raise RuntimeError(f"oracle kv read failed: {ERR[rc]}")
        return k, v

    def seed(self, k, v):
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        c = self._model.config
        n = k.size // (c.num_hidden_layers * c.kv_dim())
        rc = lib().orc_kv_seed(self._h, n, p(k), p(v))
        if rc:
            raise RuntimeError(f"oracle kv seed failed: {ERR[rc]}")
