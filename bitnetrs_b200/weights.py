"""Checkpoint ingestion: safetensors files in the layouts of
microsoft/bitnet-b1.58-2B-4T into :class:`ModelWeights` (the reference's
runtime formats, which :class:`BitNetModel` uploads).

* :func:`load_weights_from_packed` — the packed deployment checkpoint through
  the reference's canonical conversion (``convert_hf_packed_to_canonical``,
  crates/bitnet-convert/src/lib.rs:434-604): U8 projections with four logical
  rows per stored row plus a ``*_scale`` tensor each, float norms and
  embedding.
* :func:`load_weights_from_bf16` — the dense checkpoint
  (``load_weights_from_bf16``, crates/bitnet-weights/src/loader.rs:396-490):
  every projection ternarised on load by absmean.

The byte-level conversions (HF lane decode, absmean, the i8 lm_head table)
run in the native library on all host threads (bitnet_cuda_decode_hf_packed,
bitnet_cuda_absmean_ternary, bitnet_cuda_lm_head_i8_table); this module reads
the file and checks names, shapes and dtypes in the reference's order.
:func:`read_safetensors` / :func:`write_safetensors` implement the published
safetensors layout (8-byte little-endian header length, JSON header, raw
little-endian data).
"""
from __future__ import annotations

import ctypes as C
import json
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, Mapping, Tuple, Union

import numpy as np

from . import _native as N
from .errors import InvalidConfig, InvalidShape
from .model import LayerWeights, ModelConfig, ModelWeights

_NP = {"BF16": np.uint16, "F16": np.float16, "F32": np.float32, "U8": np.uint8, "I8": np.int8, "I32": np.int32,
       "F64": np.float64, "I64": np.int64, "U16": np.uint16, "I16": np.int16}


@dataclass
class Tensor:
    """One stored tensor: safetensors dtype name, shape, and its elements
    (a flat read-only view; BF16 as raw uint16 bits)."""

    dtype: str
    shape: Tuple[int, ...]
    data: np.ndarray

    def numel(self) -> int:
        """PackedTensor::numel (convert/src/lib.rs:110): product of the shape, at least 1."""
        return max(int(np.prod(self.shape, dtype=np.int64)) if self.shape else 1, 1)


def read_safetensors(path: Union[str, Path]) -> Dict[str, Tensor]:
    """Parse a safetensors file; tensor data stay memory-mapped."""
    path = Path(path)
    size = path.stat().st_size
    if size < 8:
        raise InvalidShape(f"File too small to be a valid safetensors file: {size} bytes")
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        if 8 + n > size:
            raise InvalidShape(f"safetensors header length ({n}) exceeds file size ({size})")
        header = json.loads(f.read(n))
    data = np.memmap(path, dtype=np.uint8, mode="r", offset=8 + n) if size > 8 + n else np.zeros(0, np.uint8)
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dtype, shape = meta["dtype"], tuple(int(s) for s in meta["shape"])
        b, e = (int(x) for x in meta["data_offsets"])
        if not 0 <= b <= e <= data.size:
            raise InvalidShape(f"Tensor '{name}' data offsets [{b}, {e}) exceed data region size {data.size}")
        raw = data[b:e]
        npt = _NP.get(dtype)
        out[name] = Tensor(dtype, shape, raw.view(npt) if npt is not None and raw.size % np.dtype(npt).itemsize == 0
                           else raw)
    return out


def write_safetensors(path: Union[str, Path], tensors: Mapping[str, Tuple[str, Tuple[int, ...], np.ndarray]]) -> None:
    """Write {name: (dtype, shape, array)} (arrays in the dtype's storage
    type: uint16 bits for BF16) in insertion order."""
    header, blobs, off = {}, [], 0
    for name, (dtype, shape, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


# ---------------------------------------------------------------------------
# Native conversions.
# ---------------------------------------------------------------------------
def decode_hf_packed(packed: np.ndarray, packed_rows: int, cols: int, weight_scale: float) -> np.ndarray:
    """decode_packed_projection (convert/src/lib.rs:235-325) into reference
    runtime rows: uint8 [4*packed_rows * ceil(cols/4)]."""
    src = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1)
    out = np.empty(4 * packed_rows * ((cols + 3) // 4), dtype=np.uint8)
    N.check(N.cuda_lib().bitnet_cuda_decode_hf_packed(N.ptr(src), src.size, packed_rows, cols, weight_scale,
                                                      N.ptr(out), out.size))
    return out


def absmean_ternary(w: np.ndarray, rows: int, cols: int) -> Tuple[np.ndarray, float]:
    """quantise_weight (loader.rs:1037-1070): packed runtime rows + scale."""
    src = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    if src.size != rows * cols:
        raise InvalidShape(f"[{rows}, {cols}] = {rows * cols} elements, got {src.size}")
    out = np.empty(rows * ((cols + 3) // 4), dtype=np.uint8)
    s = C.c_float()
    N.check(N.cuda_lib().bitnet_cuda_absmean_ternary(N.ptr(src), rows, cols, N.ptr(out), out.size, C.byref(s)))
    return out, float(s.value)


def lm_head_i8(embed_bf16: np.ndarray, rows: int, row_len: int) -> Tuple[np.ndarray, np.ndarray]:
    """quantize_bf16_rows_to_i8 (loader.rs:297-340): the weight-tied i8 table and scales."""
    e = np.ascontiguousarray(embed_bf16, dtype=np.uint16).reshape(-1)
    q = np.empty(rows * row_len, dtype=np.int8)
    s = np.empty(rows, dtype=np.float32)
    N.check(N.cuda_lib().bitnet_cuda_lm_head_i8_table(N.ptr(e), rows, row_len, N.ptr(q), N.ptr(s)))
    return q, s


# ---------------------------------------------------------------------------
# Tensor access in the reference's order and wording.
# ---------------------------------------------------------------------------
def _f32_bits_to_bf16(x: np.ndarray) -> np.ndarray:
    """half::bf16::from_f32: round to nearest even, NaN kept quiet."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u | 0x00400000) >> 16).astype(np.uint16), r)


def _as_f32(t: Tensor, key: str) -> np.ndarray:
    if t.dtype == "BF16":
        return (t.data.astype(np.uint32) << 16).view(np.float32)
    if t.dtype == "F16":
        return t.data.astype(np.float32)
    if t.dtype == "F32":
        return np.array(t.data, dtype=np.float32)
    raise InvalidShape(f"tensor '{key}' has unsupported float dtype '{t.dtype}'")


def _float_tensor(tensors: Mapping[str, Tensor], key: str, expected: int) -> np.ndarray:
    """load_float_tensor (convert/src/lib.rs:725-770)."""
    t = tensors.get(key)
    if t is None:
        raise InvalidShape(f"missing float tensor '{key}'")
    if t.numel() != expected:
        raise InvalidShape(f"tensor '{key}' has {t.numel()} elements, expected {expected}")
    return np.ascontiguousarray(_as_f32(t, key))


def _scalar_scale(tensors: Mapping[str, Tensor], key: str) -> float:
    """load_scalar_scale (convert/src/lib.rs:680-723): the first element."""
    t = tensors.get(key)
    if t is None:
        raise InvalidShape(f"missing scale tensor '{key}'")
    if t.dtype not in ("BF16", "F16", "F32"):
        raise InvalidShape(f"scale tensor '{key}' has unsupported dtype '{t.dtype}'")
    if t.data.size < 1:
        raise InvalidShape(f"{t.dtype} scale tensor '{key}' is too short")
    return float(_as_f32(Tensor(t.dtype, (1,), t.data[:1]), key)[0])


def _projection(tensors: Mapping[str, Tensor], key: str, rows: int, cols: int) -> Tuple[np.ndarray, float]:
    """load_and_decode_projection (convert/src/lib.rs:615-677)."""
    t = tensors.get(key)
    if t is None:
        raise InvalidShape(f"missing packed projection tensor '{key}'")
    if t.dtype not in ("U8", "I8"):
        raise InvalidShape(f"projection tensor '{key}' has dtype '{t.dtype}', expected U8/I8")
    if len(t.shape) != 2:
        raise InvalidShape(f"projection tensor '{key}' must be rank-2, got shape {list(t.shape)}")
    if t.shape[1] != cols:
        raise InvalidShape(f"projection tensor '{key}' has {t.shape[1]} columns, expected {cols}")
    if t.shape[0] * 4 != rows:
        raise InvalidShape(f"projection tensor '{key}' has packed rows {t.shape[0]}, expected logical rows {rows} "
                           "via 4x expansion")
    scale = _scalar_scale(tensors, key + "_scale")
    return decode_hf_packed(t.data.view(np.uint8), t.shape[0], cols, scale), scale


def validate_config(c: ModelConfig) -> None:
    """ModelConfig::validate (crates/bitnet-core/src/config.rs:110-150)."""
    for name in ("hidden_size", "num_attention_heads", "num_key_value_heads"):
        if getattr(c, name) == 0:
            raise InvalidConfig(f"{name} must be > 0")
    if c.hidden_size % c.num_attention_heads:
        raise InvalidConfig(f"hidden_size ({c.hidden_size}) must be divisible by num_attention_heads "
                            f"({c.num_attention_heads})")
    if c.num_attention_heads % c.num_key_value_heads:
        raise InvalidConfig(f"num_attention_heads ({c.num_attention_heads}) must be divisible by "
                            f"num_key_value_heads ({c.num_key_value_heads})")
    for name in ("vocab_size", "num_hidden_layers", "intermediate_size", "max_position_embeddings"):
        if getattr(c, name) == 0:
            raise InvalidConfig(f"{name} must be > 0")
    if not c.rope_theta > 0:
        raise InvalidConfig("rope_theta must be > 0")
    if not c.rms_norm_eps > 0:
        raise InvalidConfig("rms_norm_eps must be > 0")


def _tensors(source) -> Mapping[str, Tensor]:
    return source if isinstance(source, Mapping) else read_safetensors(source)


def _norms(tensors, base: str, cfg: ModelConfig, load):
    H, F = cfg.hidden_size, cfg.intermediate_size
    return (load(tensors, f"{base}.input_layernorm.weight", H),
            load(tensors, f"{base}.post_attention_layernorm.weight", H),
            load(tensors, f"{base}.self_attn.attn_sub_norm.weight", H),
            load(tensors, f"{base}.mlp.ffn_sub_norm.weight", F))


def load_weights_from_packed(source, cfg: ModelConfig) -> ModelWeights:
    """The packed checkpoint (a path or a read_safetensors map) through
    convert_hf_packed_to_canonical (convert/src/lib.rs:434-604)."""
    validate_config(cfg)
    t = _tensors(source)
    H, V, F, qd, kvd = cfg.hidden_size, cfg.vocab_size, cfg.intermediate_size, cfg.q_dim(), cfg.kv_dim()
    embed = _f32_bits_to_bf16(_float_tensor(t, "model.embed_tokens.weight", V * H))
    final_norm = _float_tensor(t, "model.norm.weight", H)
    layers = []
    for i in range(cfg.num_hidden_layers):
        base = f"model.layers.{i}"
        an, fn, asn, fsn = _norms(t, base, cfg, _float_tensor)
        q, sq = _projection(t, f"{base}.self_attn.q_proj.weight", qd, H)
        k, sk = _projection(t, f"{base}.self_attn.k_proj.weight", kvd, H)
        v, sv = _projection(t, f"{base}.self_attn.v_proj.weight", kvd, H)
        o, so = _projection(t, f"{base}.self_attn.o_proj.weight", H, qd)
        g, sg = _projection(t, f"{base}.mlp.gate_proj.weight", F, H)
        u, su = _projection(t, f"{base}.mlp.up_proj.weight", F, H)
        d, sd = _projection(t, f"{base}.mlp.down_proj.weight", H, F)
        layers.append(LayerWeights(q, k, v, o, g, u, d, sq, sk, sv, so, sg, su, sd, an, asn, fn, fsn))
    lm_q, lm_s = lm_head_i8(embed, V, H)
    return ModelWeights(cfg, embed, lm_q, lm_s, final_norm, layers)


def _require(tensors, key: str, expected: int) -> np.ndarray:
    """require_tensor (loader.rs:981-1030) over the float tensors of the file."""
    t = tensors.get(key)
    if t is None or t.dtype not in ("BF16", "F16", "F32"):
        raise InvalidShape(f"Required tensor '{key}' not found in safetensors file.")
    a = _as_f32(t, key)
    if a.size != expected:
        raise InvalidShape(f"Tensor '{key}' has {a.size} elements, expected {expected}")
    return np.ascontiguousarray(a)


def load_weights_from_bf16(source, cfg: ModelConfig) -> ModelWeights:
    """The dense checkpoint (a path or a read_safetensors map) through
    load_weights_from_bf16 (loader.rs:396-490): projections ternarised by
    absmean on load."""
    validate_config(cfg)
    t = _tensors(source)
    H, V, F, qd, kvd = cfg.hidden_size, cfg.vocab_size, cfg.intermediate_size, cfg.q_dim(), cfg.kv_dim()
    embed = _f32_bits_to_bf16(_require(t, "model.embed_tokens.weight", V * H))
    final_norm = _require(t, "model.norm.weight", H)
    lm_q, lm_s = lm_head_i8(embed, V, H)
    layers = []
    for i in range(cfg.num_hidden_layers):
        base = f"model.layers.{i}"
        an, fn, asn, fsn = _norms(t, base, cfg, _require)

        def proj(name, rows, cols):
            return absmean_ternary(_require(t, f"{base}.{name}.weight", rows * cols), rows, cols)

        q, sq = proj("self_attn.q_proj", qd, H)
        k, sk = proj("self_attn.k_proj", kvd, H)
        v, sv = proj("self_attn.v_proj", kvd, H)
        o, so = proj("self_attn.o_proj", H, qd)
        g, sg = proj("mlp.gate_proj", F, H)
        u, su = proj("mlp.up_proj", F, H)
        d, sd = proj("mlp.down_proj", H, F)
        layers.append(LayerWeights(q, k, v, o, g, u, d, sq, sk, sv, so, sg, su, sd, an, asn, fn, fsn))
    return ModelWeights(cfg, embed, lm_q, lm_s, final_norm, layers)


def load_model_config(path: Union[str, Path]) -> ModelConfig:
    """ModelConfig from a HuggingFace config.json (the fields the forward uses),
    with load_model_config's defaults (crates/bitnet-weights/src/config.rs:96-120):
    num_key_value_heads = num_attention_heads, rope_theta 10000, rms_norm_eps 1e-5."""
    j = json.loads(Path(path).read_text())
    return ModelConfig(int(j["vocab_size"]), int(j["hidden_size"]), int(j["num_hidden_layers"]),
                       int(j["num_attention_heads"]), int(j.get("num_key_value_heads", j["num_attention_heads"])),
                       int(j["intermediate_size"]), int(j["max_position_embeddings"]),
                       float(j.get("rope_theta", 10000.0)), float(j.get("rms_norm_eps", 1e-5)))


def detect_weight_format(path: Union[str, Path]) -> str:
    """detect_weight_format (crates/bitnet-inference/src/lib.rs:428-452):
    "packed" when any tensor of the file is U8, else "bf16" (also when the
    header cannot be read)."""
    try:
        p = Path(path)
        with open(p, "rb") as f:
            (n,) = struct.unpack("<Q", f.read(8))
            header = json.loads(f.read(n))
    except Exception:
        return "bf16"
    return "packed" if any(isinstance(m, dict) and m.get("dtype") == "U8" for k, m in header.items()
                           if k != "__metadata__") else "bf16"


def resolve_model_config(model_path: Union[str, Path]) -> ModelConfig:
    """resolve_model_config (crates/bitnet-inference/src/lib.rs:455-488): the
    sibling config.json of the checkpoint when it exists, else the 2B config."""
    from .model import bitnet_2b_config

    cfg = Path(model_path).parent / "config.json"
    return load_model_config(cfg) if cfg.exists() else bitnet_2b_config()


def load_weights(model_path: Union[str, Path], cfg: ModelConfig = None) -> ModelWeights:
    """What InferenceEngine::new does with a checkpoint
    (crates/bitnet-inference/src/lib.rs:529-580): the config from
    resolve_model_config unless given, then the packed or bf16 loader by
    detect_weight_format."""
    cfg = cfg if cfg is not None else resolve_model_config(model_path)
    if detect_weight_format(model_path) == "packed":
        return load_weights_from_packed(model_path, cfg)
    return load_weights_from_bf16(model_path, cfg)
