"""Device-resident BitNet b1.58 model on the B200 C ABI.

Python mirror of the reference's model API:

* :class:`ModelConfig`  — ``bitnet_core::config::ModelConfig`` (config.rs:26-62)
  with :func:`bitnet_2b_config` (config.rs:161-173);
* :class:`ModelWeights` — ``bitnet_weights::loader::ModelWeights`` (loader.rs:241-283)
  as numpy arrays in the reference's formats;
* :class:`BitNetModel`  — ``BitNetModel::{new, forward, forward_into, new_kv_cache}``
  (crates/bitnet-model/src/lib.rs:462-1200), weights uploaded once;
* :class:`KVCache`      — the paged device KV cache that replaces ``KVCache``
  (model/src/lib.rs:118-315); one cache serves many sequences;
* :meth:`BitNetModel.generate` — greedy ``generate_from_tokens_streaming``
  (crates/bitnet-inference/src/lib.rs:701-777).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import numpy as np

from . import _native as N
from ._native import check, ptr
from .backend import CudaBackend

KV_F32 = 0
KV_BF16 = 1
PAGE = 16
EOS_LLAMA3_EOT = 128009  # tokenizer eos_token_id() of the LLaMA-3 tokenizer
EOS_LLAMA3_TEXT = 128001  # second stop id checked by the reference generate loop


@dataclass
class ModelConfig:
    vocab_size: int
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    intermediate_size: int
    max_position_embeddings: int
    rope_theta: float
    rms_norm_eps: float

    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim()

    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim()

    def to_c(self) -> N.Config:
        return N.Config(self.vocab_size, self.hidden_size, self.num_hidden_layers, self.num_attention_heads,
                        self.num_key_value_heads, self.intermediate_size, self.max_position_embeddings,
                        self.rope_theta, self.rms_norm_eps)


def bitnet_2b_config() -> ModelConfig:
    """BitNet b1.58 2B-4T (crates/bitnet-core/src/config.rs:161-173)."""
    return ModelConfig(128_256, 2560, 30, 20, 5, 6912, 4096, 500_000.0, 1e-5)


def scaled_model_config() -> ModelConfig:
    """The larger shape served tensor-parallel: hidden 4096, 32 layers, 32
    query / 8 KV heads of 128, intermediate 14336, the 2B vocabulary, RoPE
    theta and eps (the 2B family's layer structure at Llama-3-8B widths)."""
    return ModelConfig(128_256, 4096, 32, 32, 8, 14336, 4096, 500_000.0, 1e-5)


def tiny_config() -> ModelConfig:
    """The reference's unit-test model (crates/bitnet-model/src/lib.rs:1267-1279)."""
    return ModelConfig(16, 8, 2, 2, 1, 16, 32, 10000.0, 1e-5)


@dataclass
class LayerWeights:
    """Packed projections (uint8, ``rows*ceil(cols/4)``) + per-tensor scales + f32 norms."""

    q_proj: np.ndarray
    k_proj: np.ndarray
    v_proj: np.ndarray
    o_proj: np.ndarray
    gate_proj: np.ndarray
    up_proj: np.ndarray
    down_proj: np.ndarray
    q_scale: float
    k_scale: float
    v_scale: float
    o_scale: float
    gate_scale: float
    up_scale: float
    down_scale: float
    attention_norm: np.ndarray
    attn_sub_norm: np.ndarray
    ffn_norm: np.ndarray
    ffn_sub_norm: np.ndarray


@dataclass
class ModelWeights:
    config: ModelConfig
    embed_tokens: np.ndarray  # uint16 bf16 bits [V*H]
    lm_head_i8: np.ndarray  # int8 [V*H]
    lm_head_scales: np.ndarray  # f32 [V]
    final_norm: np.ndarray  # f32 [H]
    layers: List[LayerWeights] = field(default_factory=list)


def _c_weights(w: ModelWeights):
    layers = (N.LayerWeights * len(w.layers))()
    for i, L in enumerate(w.layers):
        layers[i] = N.LayerWeights(
            ptr(L.q_proj), ptr(L.k_proj), ptr(L.v_proj), ptr(L.o_proj), ptr(L.gate_proj), ptr(L.up_proj),
            ptr(L.down_proj), L.q_scale, L.k_scale, L.v_scale, L.o_scale, L.gate_scale, L.up_scale, L.down_scale,
            ptr(L.attention_norm), ptr(L.attn_sub_norm), ptr(L.ffn_norm), ptr(L.ffn_sub_norm))
    cw = N.Weights(ptr(w.embed_tokens), ptr(w.lm_head_i8), ptr(w.lm_head_scales), ptr(w.final_norm), layers)
    return cw, layers


def _check_weights(w: ModelWeights) -> None:
    c = w.config
    H, F, V, qd, kvd = c.hidden_size, c.intermediate_size, c.vocab_size, c.q_dim(), c.kv_dim()
    pc = lambda k: (k + 3) // 4  # noqa: E731
    if len(w.layers) != c.num_hidden_layers:
        raise ValueError("layer count does not match config")
    for L in w.layers:
        for name, arr, n in (("q_proj", L.q_proj, qd * pc(H)), ("k_proj", L.k_proj, kvd * pc(H)),
                             ("v_proj", L.v_proj, kvd * pc(H)), ("o_proj", L.o_proj, H * pc(qd)),
                             ("gate_proj", L.gate_proj, F * pc(H)), ("up_proj", L.up_proj, F * pc(H)),
                             ("down_proj", L.down_proj, H * pc(F))):
            if arr.dtype != np.uint8 or arr.size != n or not arr.flags.c_contiguous:
                raise ValueError(f"{name}: expected {n} packed uint8 bytes")
        for name, arr, n in (("attention_norm", L.attention_norm, H), ("attn_sub_norm", L.attn_sub_norm, qd),
                             ("ffn_norm", L.ffn_norm, H), ("ffn_sub_norm", L.ffn_sub_norm, F)):
            if arr.dtype != np.float32 or arr.size != n or not arr.flags.c_contiguous:
                raise ValueError(f"{name}: expected {n} float32 values")
    if w.embed_tokens.dtype != np.uint16 or w.embed_tokens.size != V * H:
        raise ValueError("embed_tokens: expected V*H bf16 (uint16) values")
    if w.lm_head_i8.dtype != np.int8 or w.lm_head_i8.size != V * H:
        raise ValueError("lm_head_i8: expected V*H int8 values")
    if w.lm_head_scales.dtype != np.float32 or w.lm_head_scales.size != V:
        raise ValueError("lm_head_scales: expected V float32 values")
    if w.final_norm.dtype != np.float32 or w.final_norm.size != H:
        raise ValueError("final_norm: expected H float32 values")


class BitNetModel:
    """Weights resident on one GPU; forward passes run entirely on the device."""

    def __init__(self, weights: ModelWeights, backend: Optional[CudaBackend] = None, max_batch_tokens: int = 4096,
                 tp=None):
        """`tp` (a :class:`bitnetrs_b200.tp.TensorParallel`) makes this a
        tensor-parallel shard: `weights` is the full model, the device keeps
        this rank's share, and every rank must run the same calls together."""
        _check_weights(weights)
        self.backend = backend if backend is not None else CudaBackend(0)
        self.config = weights.config
        self.tp = tp
        self._lib = N.cuda_lib()
        cw, keep = _c_weights(weights)
        cfg = weights.config.to_c()
        h = C.c_void_p()
        if tp is None:
            check(self._lib.bitnet_cuda_model_create(self.backend.handle, C.byref(cfg), C.byref(cw),
                                                     max_batch_tokens, C.byref(h)))
        else:
            uid = (C.c_uint8 * len(tp.unique_id)).from_buffer_copy(tp.unique_id)
            check(self._lib.bitnet_cuda_model_create_tp(self.backend.handle, C.byref(cfg), C.byref(cw),
                                                        max_batch_tokens, tp.rank, tp.world, uid, len(tp.unique_id),
                                                        C.byref(h)))
        self._h = h
        self.max_batch_tokens = max_batch_tokens

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            self._lib.bitnet_cuda_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def new_kv_cache(self, num_pages: int, max_seqs: int = 1, kv_dtype: int = KV_F32) -> "KVCache":
        return KVCache(self, num_pages, max_seqs, kv_dtype)

    # BitNetModel::forward_into for one sequence.
    def forward_into(self, tokens: Sequence[int], start_pos: int, kv: "KVCache", output_logits: np.ndarray,
                     seq: int = 0) -> None:
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        if output_logits.dtype != np.float32 or output_logits.size != self.config.vocab_size:
            raise ValueError("output_logits must be float32 of length vocab_size")
        check(self._lib.bitnet_cuda_forward(self._h, kv.handle, seq, ptr(t), t.size, start_pos, ptr(output_logits)))

    def forward(self, tokens: Sequence[int], start_pos: int, kv: "KVCache", seq: int = 0) -> np.ndarray:
        out = np.empty(self.config.vocab_size, dtype=np.float32)
        self.forward_into(tokens, start_pos, kv, out, seq)
        return out

    def decode_step(self, kv: "KVCache", seq_ids, tokens, want_logits: bool = False):
        """One new token for each listed sequence; returns (next_tokens, logits or None)."""
        s = np.ascontiguousarray(np.asarray(seq_ids, dtype=np.uint32))
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        if s.size != t.size:
            raise ValueError("seq_ids and tokens must have the same length")
        nxt = np.empty(s.size, dtype=np.uint32)
        logits = np.empty((s.size, self.config.vocab_size), dtype=np.float32) if want_logits else None
        check(self._lib.bitnet_cuda_decode_step(self._h, kv.handle, s.size, ptr(s), ptr(t), ptr(logits), ptr(nxt)))
        return nxt, logits

    def decode_step_device(self, kv: "KVCache", seq_ids, d_tokens: int, d_next: int, d_logits: int = 0,
                           stream: int = 0) -> None:
        """Device-resident decode step; d_* are device addresses (e.g. torch ``data_ptr()``)."""
        s = np.ascontiguousarray(np.asarray(seq_ids, dtype=np.uint32))
        check(self._lib.bitnet_cuda_decode_step_device(self._h, kv.handle, s.size, ptr(s), d_tokens, d_next,
                                                       d_logits or None, stream or None))

    def prefill(self, kv: "KVCache", seq_ids, token_lists, want_logits: bool = False):
        """Ragged prefill: token_lists[i] is appended to sequence seq_ids[i]."""
        s = np.ascontiguousarray(np.asarray(seq_ids, dtype=np.uint32))
        lens = [len(x) for x in token_lists]
        cu = np.zeros(len(lens) + 1, dtype=np.uint32)
        cu[1:] = np.cumsum(lens)
        toks = np.ascontiguousarray(np.concatenate([np.asarray(x, dtype=np.uint32) for x in token_lists]))
        nxt = np.empty(s.size, dtype=np.uint32)
        logits = np.empty((s.size, self.config.vocab_size), dtype=np.float32) if want_logits else None
        check(self._lib.bitnet_cuda_prefill(self._h, kv.handle, s.size, ptr(s), ptr(toks), ptr(cu), ptr(logits),
                                            ptr(nxt)))
        return nxt, logits

    def prefill_packed(self, kv: "KVCache", seq_ids, token_lists, want_logits: bool = False):
        """Ragged prefill of any number of prompt tokens: the prompts are packed
        into steps of at most ``max_batch_tokens`` (batching.pack_steps) and run
        in order. Returns, per sequence, the greedy next token and (optionally)
        the logits after its last prompt token; an empty prompt gets
        next token 0 and zero logits."""
        from .batching import pack_steps

        seq_ids = [int(x) for x in seq_ids]
        if len(seq_ids) != len(token_lists):
            raise ValueError("seq_ids and token_lists must have the same length")
        lens = [len(x) for x in token_lists]
        nxt = np.zeros(len(seq_ids), dtype=np.uint32)
        logits = np.zeros((len(seq_ids), self.config.vocab_size), dtype=np.float32) if want_logits else None
        for step in pack_steps(lens, self.max_batch_tokens):
            n, lg = self.prefill(kv, [seq_ids[i] for i, _, _ in step],
                                 [np.asarray(token_lists[i])[a:a + c] for i, a, c in step], want_logits)
            for j, (i, a, c) in enumerate(step):
                if a + c == lens[i]:  # the prompt's last chunk
                    nxt[i] = n[j]
                    if want_logits:
                        logits[i] = lg[j]
        return nxt, logits

    def check(self) -> None:
        check(self._lib.bitnet_cuda_model_check(self._h))

    NUMERICS = {"auto": 0, "exact": 1, "fast": 2}

    def set_numerics(self, mode: str) -> None:
        """"auto" (reference-order kernels for steps <= 16 tokens), "exact" or "fast"."""
        check(self._lib.bitnet_cuda_model_set_numerics(self._h, self.NUMERICS[mode]))

    KERNEL_CLASSES = ("attention", "ternary_matmul", "norm_quant", "rope_kv_store", "lm_head", "other",
                      "decode_layers")

    def set_fused_decode(self, enable: bool) -> None:
        """One-token steps as one persistent kernel over all layers (default on
        where the model and cache fit it); off selects the per-layer kernels."""
        check(self._lib.bitnet_cuda_model_set_fused_decode(self._h, 1 if enable else 0))

    def set_kernel_timing(self, enable: bool) -> None:
        """Record CUDA events around every kernel of decode graphs captured from now on."""
        check(self._lib.bitnet_cuda_model_set_kernel_timing(self._h, 1 if enable else 0))

    def attention_kernel(self, kv: "KVCache", tokens: int = 1) -> str:
        """Name of the attention kernel a step of `tokens` query tokens over `kv` launches."""
        buf = C.create_string_buffer(64)
        check(self._lib.bitnet_cuda_model_attention_kernel(self._h, kv.handle, tokens, buf, 64))
        return buf.value.decode()

    def kernel_times(self):
        """{class: (device ms summed over the most recent timed step, launches)}."""
        ms = np.zeros(len(self.KERNEL_CLASSES), dtype=np.float32)
        n = np.zeros(len(self.KERNEL_CLASSES), dtype=np.int32)
        check(self._lib.bitnet_cuda_model_kernel_times(self._h, ptr(ms), ptr(n)))
        return {c: (float(ms[i]), int(n[i])) for i, c in enumerate(self.KERNEL_CLASSES)}

    def generate(self, kv: "KVCache", prompt: Sequence[int], max_new_tokens: int, seq: int = 0,
                 eos_ids=(EOS_LLAMA3_EOT, EOS_LLAMA3_TEXT), sampling=None) -> List[int]:
        """generate_from_tokens_streaming (crates/bitnet-inference/src/lib.rs:701-777):
        greedy without `sampling`, else sample_next_token on the device with
        that SamplingConfig (validated like SamplingConfig::validate)."""
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        out = np.empty(max(1, max_new_tokens), dtype=np.uint32)
        n = C.c_size_t()
        if sampling is None:
            check(self._lib.bitnet_cuda_generate(self._h, kv.handle, seq, ptr(p), p.size, max_new_tokens,
                                                 eos_ids[0], eos_ids[1], ptr(out), C.byref(n)))
        else:
            check(self._lib.bitnet_cuda_generate_sampled(self._h, kv.handle, seq, ptr(p), p.size, max_new_tokens,
                                                         C.byref(sampling.to_c()), eos_ids[0], eos_ids[1], ptr(out),
                                                         C.byref(n)))
        return out[: n.value].tolist()


class KVCache:
    """Paged KV cache: ``num_pages`` pages of 16 positions (all layers) shared by ``max_seqs`` sequences."""

    def __init__(self, model: BitNetModel, num_pages: int, max_seqs: int = 1, kv_dtype: int = KV_F32):
        self.model = model
        self._lib = N.cuda_lib()
        h = C.c_void_p()
        check(self._lib.bitnet_cuda_kv_create(model.handle, num_pages, max_seqs, kv_dtype, C.byref(h)))
        self._h = h
        self.kv_dtype = kv_dtype

    @property
    def handle(self):
        return self._h

    def close(self):
        if getattr(self, "_h", None):
            self._lib.bitnet_cuda_kv_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def clear(self, seq: int = 0) -> None:
        check(self._lib.bitnet_cuda_kv_seq_reset(self._h, seq))

    def len(self, seq: int = 0) -> int:
        n = C.c_size_t()
        check(self._lib.bitnet_cuda_kv_seq_len(self._h, seq, C.byref(n)))
        return n.value

    def free_pages(self) -> int:
        n = C.c_size_t()
        check(self._lib.bitnet_cuda_kv_free_pages(self._h, C.byref(n)))
        return n.value

    def reserve(self, seq: int, length: int) -> None:
        check(self._lib.bitnet_cuda_kv_seq_reserve(self._h, seq, length))

    def write(self, seq: int, k: np.ndarray, v: np.ndarray) -> None:
        """Seed positions [0, n) from f32 arrays laid out [layer][pos][kv_heads*head_dim]."""
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        c = self.model.config
        n = k.size // (c.num_hidden_layers * c.kv_dim())
        if k.size != n * c.num_hidden_layers * c.kv_dim() or v.size != k.size:
            raise ValueError("k/v must be [layers][n][kv_dim]")
        check(self._lib.bitnet_cuda_kv_seq_write(self._h, seq, n, ptr(k), ptr(v)))

    def read(self, seq: int, n: int):
        c = self.model.config
        k = np.empty((c.num_hidden_layers, n, c.kv_dim()), dtype=np.float32)
        v = np.empty_like(k)
        check(self._lib.bitnet_cuda_kv_seq_read(self._h, seq, n, ptr(k), ptr(v)))
        return k, v

    def fill_random(self, seq: int, n: int, seed: int) -> None:
        check(self._lib.bitnet_cuda_kv_seq_fill_random(self._h, seq, n, seed))


def kernel_launches() -> int:
    return int(N.cuda_lib().bitnet_cuda_kernel_launches(None))
