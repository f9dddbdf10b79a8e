"""ctypes bindings of ``include/bitnet_cuda.h`` (libbitnet_cuda.so) and of the
seeded input generator (libbitnet_synth.so).

The libraries are built in-tree by ``python -m bitnetrs_b200.build``.  Loading
fails loudly when they are missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

PKG = Path(__file__).resolve().parent
CUDA_LIB_PATH = PKG / "libbitnet_cuda.so"
SYNTH_LIB_PATH = PKG / "libbitnet_synth.so"

vp = C.c_void_p
sz = C.c_size_t
f32 = C.c_float
u32 = C.c_uint32
i32 = C.c_int
u64 = C.c_uint64
P_ctx = C.c_void_p


class Config(C.Structure):
    """bitnet_cuda_config == ModelConfig (crates/bitnet-core/src/config.rs:26-62)."""

    _fields_ = [
        ("vocab_size", u32),
        ("hidden_size", u32),
        ("num_hidden_layers", u32),
        ("num_attention_heads", u32),
        ("num_key_value_heads", u32),
        ("intermediate_size", u32),
        ("max_position_embeddings", u32),
        ("rope_theta", f32),
        ("rms_norm_eps", f32),
    ]


class Sampling(C.Structure):
    """bitnet_cuda_sampling == SamplingConfig (crates/bitnet-inference/src/lib.rs:80-112)."""

    _fields_ = [("temperature", f32), ("top_p", f32), ("top_k", u32), ("repetition_penalty", f32), ("seed", u64)]


class LayerWeights(C.Structure):
    """bitnet_cuda_layer_weights == LayerWeights (crates/bitnet-weights/src/loader.rs:121-203)."""

    _fields_ = [
        ("q_proj", vp), ("k_proj", vp), ("v_proj", vp), ("o_proj", vp),
        ("gate_proj", vp), ("up_proj", vp), ("down_proj", vp),
        ("q_scale", f32), ("k_scale", f32), ("v_scale", f32), ("o_scale", f32),
        ("gate_scale", f32), ("up_scale", f32), ("down_scale", f32),
        ("attention_norm", vp), ("attn_sub_norm", vp), ("ffn_norm", vp), ("ffn_sub_norm", vp),
    ]


class Weights(C.Structure):
    """bitnet_cuda_weights == ModelWeights (loader.rs:241-283)."""

    _fields_ = [
        ("embed_tokens", vp),
        ("lm_head_i8", vp),
        ("lm_head_scales", vp),
        ("final_norm", vp),
        ("layers", C.POINTER(LayerWeights)),
    ]


# name: (restype, [argtypes])
_CUDA_SIGS = {
    "bitnet_cuda_create": (i32, [u32, C.POINTER(vp)]),
    "bitnet_cuda_destroy": (None, [vp]),
    "bitnet_cuda_device_name": (C.c_char_p, [vp]),
    "bitnet_cuda_last_error": (C.c_char_p, []),
    "bitnet_cuda_last_error_expected": (C.c_char_p, []),
    "bitnet_cuda_last_error_got": (C.c_char_p, []),
    "bitnet_cuda_kernel_binary_version": (i32, [vp]),
    "bitnet_cuda_version": (C.c_char_p, []),
    "bitnet_cuda_ternary_gemv": (i32, [vp, vp, sz, f32, vp, sz, vp, sz, sz, sz]),
    "bitnet_cuda_ternary_gemv_with_activation_quant": (i32, [vp, vp, sz, f32, vp, sz, vp, sz, sz, sz]),
    "bitnet_cuda_rms_norm": (i32, [vp, vp, sz, vp, sz, f32, vp, sz]),
    "bitnet_cuda_rope_embed": (i32, [vp, vp, sz, vp, sz, sz, sz, sz, sz, f32]),
    "bitnet_cuda_masked_attention": (i32, [vp, vp, sz, vp, sz, vp, sz, vp, sz, sz, sz, sz, sz]),
    "bitnet_cuda_squared_relu": (i32, [vp, vp, sz]),
    "bitnet_cuda_softmax": (i32, [vp, vp, sz]),
    "bitnet_cuda_elementwise_mul": (i32, [vp, vp, sz, vp, sz, vp, sz]),
    "bitnet_cuda_lm_head_matmul_into": (i32, [vp, vp, sz, vp, sz, vp, sz, sz, sz]),
    "bitnet_cuda_lm_head_matmul_bf16_into": (i32, [vp, vp, sz, vp, sz, vp, sz, sz, sz]),
    "bitnet_cuda_sqrelu_gate": (i32, [vp, vp, sz, vp, sz, vp, sz]),
    "bitnet_cuda_ternary_gemv_preq": (i32, [vp, vp, sz, f32, vp, sz, f32, vp, sz, sz, sz]),
    "bitnet_cuda_lm_head_matmul_i8_into": (i32, [vp, vp, sz, vp, sz, vp, sz, vp, sz, sz, sz]),
    "bitnet_cuda_absmax_quantize_row": (i32, [vp, vp, sz, vp, sz, C.POINTER(f32)]),
    "bitnet_cuda_ternary_gemv_preq_acc": (i32, [vp, vp, sz, f32, vp, sz, f32, vp, sz, vp, sz, sz]),
    "bitnet_cuda_greedy_argmax": (i32, [vp, vp, sz, C.POINTER(u32)]),
    "bitnet_cuda_sample_next_token": (i32, [vp, vp, sz, C.POINTER(Sampling), vp, sz, C.POINTER(u32)]),
    "bitnet_cuda_weight_upload": (i32, [vp, vp, sz, sz, sz, f32, C.POINTER(vp)]),
    "bitnet_cuda_weight_destroy": (None, [vp]),
    "bitnet_cuda_quantize_rows_device": (i32, [vp, vp, i32, sz, sz, vp, sz, vp, vp, vp, vp]),
    "bitnet_cuda_ternary_matmul_device": (i32, [vp, vp, vp, sz, vp, vp, sz, vp, vp, vp]),
    "bitnet_cuda_model_create": (i32, [vp, C.POINTER(Config), C.POINTER(Weights), u32, C.POINTER(vp)]),
    "bitnet_cuda_model_destroy": (None, [vp]),
    "bitnet_cuda_decode_hf_packed": (i32, [vp, sz, sz, sz, f32, vp, sz]),
    "bitnet_cuda_absmean_ternary": (i32, [vp, sz, sz, vp, sz, C.POINTER(f32)]),
    "bitnet_cuda_lm_head_i8_table": (i32, [vp, sz, sz, vp, vp]),
    "bitnet_cuda_tp_unique_id": (i32, [vp, sz]),
    "bitnet_cuda_model_create_tp": (i32, [vp, C.POINTER(Config), C.POINTER(Weights), u32, u32, u32, vp, sz,
                                          C.POINTER(vp)]),
    "bitnet_cuda_kv_create": (i32, [vp, u32, u32, i32, C.POINTER(vp)]),
    "bitnet_cuda_kv_destroy": (None, [vp]),
    "bitnet_cuda_kv_seq_reset": (i32, [vp, u32]),
    "bitnet_cuda_kv_seq_len": (i32, [vp, u32, C.POINTER(sz)]),
    "bitnet_cuda_kv_free_pages": (i32, [vp, C.POINTER(sz)]),
    "bitnet_cuda_kv_seq_write": (i32, [vp, u32, sz, vp, vp]),
    "bitnet_cuda_kv_seq_read": (i32, [vp, u32, sz, vp, vp]),
    "bitnet_cuda_kv_seq_fill_random": (i32, [vp, u32, sz, u64]),
    "bitnet_cuda_kv_seq_reserve": (i32, [vp, u32, sz]),
    "bitnet_cuda_forward": (i32, [vp, vp, u32, vp, sz, sz, vp]),
    "bitnet_cuda_decode_step": (i32, [vp, vp, sz, vp, vp, vp, vp]),
    "bitnet_cuda_decode_step_device": (i32, [vp, vp, sz, vp, vp, vp, vp, vp]),
    "bitnet_cuda_prefill": (i32, [vp, vp, sz, vp, vp, vp, vp, vp]),
    "bitnet_cuda_generate": (i32, [vp, vp, u32, vp, sz, sz, u32, u32, vp, C.POINTER(sz)]),
    "bitnet_cuda_generate_sampled": (i32, [vp, vp, u32, vp, sz, sz, C.POINTER(Sampling), u32, u32, vp,
                                           C.POINTER(sz)]),
    "bitnet_cuda_model_check": (i32, [vp]),
    "bitnet_cuda_ternary_gemv_quant_noalloc": (i32, [vp, vp, vp, sz, vp, sz, vp]),
    "bitnet_cuda_model_attention_kernel": (i32, [vp, vp, u32, vp, sz]),
    "bitnet_cuda_model_set_numerics": (i32, [vp, i32]),
    "bitnet_cuda_model_set_kernel_timing": (i32, [vp, i32]),
    "bitnet_cuda_model_kernel_times": (i32, [vp, vp, vp]),
    "bitnet_cuda_model_set_fused_decode": (i32, [vp, i32]),
    "bitnet_cuda_kernel_launches": (u64, [vp]),
}

_SYNTH_SIGS = {
    "synth_set_threads": (i32, [i32]),
    "synth_normal_f32": (None, [u64, u64, u64, sz, f32, vp]),
    "synth_bf16_normal": (None, [u64, u64, sz, f32, vp]),
    "synth_ternary_absmean": (i32, [u64, u64, sz, sz, f32, vp, C.POINTER(f32)]),
    "synth_ternary_codes": (None, [u64, u64, sz, sz, C.c_double, C.c_double, vp]),
    "synth_quantize_bf16_rows_to_i8": (None, [vp, sz, sz, vp, vp]),
    "synth_uniform_u32": (None, [u64, u64, sz, u32, u32, vp]),
    "synth_kv_normal": (None, [u64, u32, u32, u32, u32, sz, vp, vp]),
}

_cuda = None
_synth = None


def _bind(lib, sigs):
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def cuda_lib():
    """The CUDA backend library; raises if it has not been built."""
    global _cuda
    if _cuda is None:
        if not CUDA_LIB_PATH.exists():
            raise RuntimeError(
                f"{CUDA_LIB_PATH} is missing: build it with `python -m bitnetrs_b200.build` "
                "(the backend has no CPU fallback)")
        lib = C.CDLL(str(CUDA_LIB_PATH))
        _bind(lib, _CUDA_SIGS)
        _cuda = lib
    return _cuda


def synth_lib():
    global _synth
    if _synth is None:
        if not SYNTH_LIB_PATH.exists():
            raise RuntimeError(f"{SYNTH_LIB_PATH} is missing: build it with `python -m bitnetrs_b200.build`")
        lib = C.CDLL(str(SYNTH_LIB_PATH))
        _bind(lib, _SYNTH_SIGS)
        _synth = lib
    return _synth


def exported_cuda_symbols():
    return list(_CUDA_SIGS)


def ptr(a):
    """Data pointer of a numpy array (or None)."""
    return None if a is None else a.ctypes.data


def check(code: int) -> None:
    if code != 0:
        from .errors import raise_for
        lib = cuda_lib()
        msg = lib.bitnet_cuda_last_error().decode(errors="replace")
        raise_for(code, msg, lib.bitnet_cuda_last_error_expected().decode(errors="replace"),
                  lib.bitnet_cuda_last_error_got().decode(errors="replace"))
