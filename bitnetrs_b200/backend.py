"""CudaBackend — the Backend trait of bitnetrs on the B200 C ABI.

Method names, argument meaning, in-place semantics and error variants follow
``trait Backend`` (crates/bitnet-core/src/backend/mod.rs:128-517) and its CPU
implementation (crates/bitnet-cpu/src/lib.rs:158-585): read-only slices are
numpy arrays, ``&mut [T]`` outputs are caller-allocated numpy arrays that the
call overwrites, and errors raise the ``BitNetError`` subclasses of
:mod:`bitnetrs_b200.errors`.  Every call runs on the GPU; there is no CPU
fallback.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from ._native import check, ptr


def _arr(a, dtype):
    a = np.asarray(a)
    if a.dtype != dtype:
        raise TypeError(f"expected {np.dtype(dtype)} array, got {a.dtype}")
    if not a.flags.c_contiguous:
        raise TypeError("arrays must be C-contiguous")
    return a


def _out(a, dtype):
    if not isinstance(a, np.ndarray) or a.dtype != dtype or not a.flags.c_contiguous or not a.flags.writeable:
        raise TypeError(f"output must be a writeable C-contiguous {np.dtype(dtype)} numpy array")
    return a


class CudaBackend:
    """One CUDA context on one GPU (``Device::Gpu { device_id }``)."""

    def __init__(self, device_id: int = 0):
        self._lib = N.cuda_lib()
        h = C.c_void_p()
        check(self._lib.bitnet_cuda_create(device_id, C.byref(h)))
        self._h = h
        self.device_id = device_id

    # -- lifecycle ------------------------------------------------------------
    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            self._lib.bitnet_cuda_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def device_name(self) -> str:
        return self._lib.bitnet_cuda_device_name(self._h).decode()

    # -- core linear algebra ----------------------------------------------------
    def ternary_gemv(self, weight_packed, weight_scale, input, output, out_features, in_features):
        w, x, o = _arr(weight_packed, np.uint8), _arr(input, np.float32), _out(output, np.float32)
        check(self._lib.bitnet_cuda_ternary_gemv(self._h, ptr(w), w.size, weight_scale, ptr(x), x.size, ptr(o), o.size,
                                                 out_features, in_features))

    def ternary_gemv_with_activation_quant(self, weight_packed, weight_scale, input, output, out_features,
                                           in_features):
        w, x, o = _arr(weight_packed, np.uint8), _arr(input, np.float32), _out(output, np.float32)
        check(self._lib.bitnet_cuda_ternary_gemv_with_activation_quant(
            self._h, ptr(w), w.size, weight_scale, ptr(x), x.size, ptr(o), o.size, out_features, in_features))

    def ternary_gemv_preq(self, weight_packed, weight_scale, activation_q, act_absmax, output, out_features,
                          in_features, acc=None):
        """``acc`` (optional int32 array) receives the exact integer accumulators."""
        w, x, o = _arr(weight_packed, np.uint8), _arr(activation_q, np.int8), _out(output, np.float32)
        if acc is None:
            check(self._lib.bitnet_cuda_ternary_gemv_preq(self._h, ptr(w), w.size, weight_scale, ptr(x), x.size,
                                                          act_absmax, ptr(o), o.size, out_features, in_features))
        else:
            a = _out(acc, np.int32)
            if a.size != o.size:
                raise ValueError("acc must have out_features elements")
            check(self._lib.bitnet_cuda_ternary_gemv_preq_acc(self._h, ptr(w), w.size, weight_scale, ptr(x), x.size,
                                                              act_absmax, ptr(o), o.size, ptr(a), out_features,
                                                              in_features))

    # -- normalisation / positional encoding / attention -----------------------------
    def rms_norm(self, input, weight, eps, output):
        x, w, o = _arr(input, np.float32), _arr(weight, np.float32), _out(output, np.float32)
        check(self._lib.bitnet_cuda_rms_norm(self._h, ptr(x), x.size, ptr(w), w.size, eps, ptr(o), o.size))

    def rope_embed(self, q, k, position, head_dim, n_heads, n_kv_heads, theta):
        q, k = _out(q, np.float32), _out(k, np.float32)
        check(self._lib.bitnet_cuda_rope_embed(self._h, ptr(q), q.size, ptr(k), k.size, position, head_dim, n_heads,
                                               n_kv_heads, theta))

    def masked_attention(self, q, k_cache, v_cache, output, n_heads, n_kv_heads, head_dim, cur_pos):
        q, k, v, o = (_arr(q, np.float32), _arr(k_cache, np.float32), _arr(v_cache, np.float32),
                      _out(output, np.float32))
        check(self._lib.bitnet_cuda_masked_attention(self._h, ptr(q), q.size, ptr(k), k.size, ptr(v), v.size, ptr(o),
                                                     o.size, n_heads, n_kv_heads, head_dim, cur_pos))

    # -- activations / elementwise ---------------------------------------------------
    def squared_relu(self, x):
        x = _out(x, np.float32)
        check(self._lib.bitnet_cuda_squared_relu(self._h, ptr(x), x.size))

    def softmax(self, x):
        x = _out(x, np.float32)
        check(self._lib.bitnet_cuda_softmax(self._h, ptr(x), x.size))

    def elementwise_mul(self, a, b, out):
        a, b, o = _arr(a, np.float32), _arr(b, np.float32), _out(out, np.float32)
        check(self._lib.bitnet_cuda_elementwise_mul(self._h, ptr(a), a.size, ptr(b), b.size, ptr(o), o.size))

    def sqrelu_gate(self, gate, up, out):
        g, u, o = _arr(gate, np.float32), _arr(up, np.float32), _out(out, np.float32)
        check(self._lib.bitnet_cuda_sqrelu_gate(self._h, ptr(g), g.size, ptr(u), u.size, ptr(o), o.size))

    # -- lm_head -----------------------------------------------------------------------
    def lm_head_matmul_into(self, hidden, weights, output, vocab_size, hidden_size):
        h, w, o = _arr(hidden, np.float32), _arr(weights, np.float32), _out(output, np.float32)
        check(self._lib.bitnet_cuda_lm_head_matmul_into(self._h, ptr(h), h.size, ptr(w), w.size, ptr(o), o.size,
                                                        vocab_size, hidden_size))

    def lm_head_matmul_bf16_into(self, hidden, weights_bf16, output, vocab_size, hidden_size):
        """``weights_bf16``: uint16 array of raw bf16 bit patterns."""
        h, w, o = _arr(hidden, np.float32), _arr(weights_bf16, np.uint16), _out(output, np.float32)
        check(self._lib.bitnet_cuda_lm_head_matmul_bf16_into(self._h, ptr(h), h.size, ptr(w), w.size, ptr(o), o.size,
                                                             vocab_size, hidden_size))

    def lm_head_matmul_i8_into(self, hidden, weights_i8, scales, output, vocab_size, hidden_size):
        h, w, s, o = (_arr(hidden, np.float32), _arr(weights_i8, np.int8), _arr(scales, np.float32),
                      _out(output, np.float32))
        check(self._lib.bitnet_cuda_lm_head_matmul_i8_into(self._h, ptr(h), h.size, ptr(w), w.size, ptr(s), s.size,
                                                           ptr(o), o.size, vocab_size, hidden_size))

    # -- helpers the model calls outside the trait ------------------------------------------
    def absmax_quantize_row_into(self, x, out):
        """absmax_quantize_row_into (crates/bitnet-core/src/quant/absmax.rs:127-165); returns the scale."""
        x, o = _arr(x, np.float32), _out(out, np.int8)
        s = C.c_float()
        check(self._lib.bitnet_cuda_absmax_quantize_row(self._h, ptr(x), x.size, ptr(o), o.size, C.byref(s)))
        return s.value

    def greedy_argmax(self, logits) -> int:
        """Greedy sample_next_token (crates/bitnet-inference/src/lib.rs:263-274)."""
        x = _arr(logits, np.float32)
        t = C.c_uint32()
        check(self._lib.bitnet_cuda_greedy_argmax(self._h, ptr(x), x.size, C.byref(t)))
        return t.value

    def sample_next_token(self, logits: np.ndarray, config, past_tokens=()) -> int:
        """sample_next_token (crates/bitnet-inference/src/lib.rs:236-390) on the
        GPU.  `logits` (float32, C-contiguous) is modified in place as the
        reference modifies it; `config` is a SamplingConfig."""
        if logits.dtype != np.float32 or not logits.flags.c_contiguous:
            raise ValueError("logits must be a C-contiguous float32 array")
        pa = np.ascontiguousarray(np.asarray(past_tokens, dtype=np.uint32))
        t = C.c_uint32()
        check(self._lib.bitnet_cuda_sample_next_token(self._h, ptr(logits), logits.size, C.byref(config.to_c()),
                                                      ptr(pa) if pa.size else None, pa.size, C.byref(t)))
        return t.value
