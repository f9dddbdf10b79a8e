"""bitnetrs_b200 — B200 (sm_100a) backend for the bitnetrs ternary inference hot path.

The product is ``libbitnet_cuda.so`` (hand-written CUDA kernels behind the C ABI
of ``include/bitnet_cuda.h``).  This package is its Python host mirror:

* :class:`CudaBackend` — the reference ``Backend`` trait (host slices);
* :class:`BitNetModel` / :class:`KVCache` — device-resident model, paged KV
  cache, batched decode / prefill, greedy and sampled generate;
* :mod:`bitnetrs_b200.tp` — tensor-parallel shards over NCCL (one process per GPU);
* :mod:`bitnetrs_b200.synth` — seeded synthetic models in the reference formats.
"""
from .backend import CudaBackend
from .errors import BackendError, BitNetError, InvalidConfig, InvalidShape, QuantizationError
from .model import (KV_BF16, KV_F32, BitNetModel, KVCache, LayerWeights, ModelConfig, ModelWeights,
                    bitnet_2b_config, kernel_launches, scaled_model_config, tiny_config)

__all__ = [
    "CudaBackend", "BitNetModel", "KVCache", "ModelConfig", "ModelWeights", "LayerWeights", "bitnet_2b_config",
    "scaled_model_config",
    "tiny_config", "KV_F32", "KV_BF16", "BitNetError", "InvalidShape", "QuantizationError", "BackendError",
    "InvalidConfig", "kernel_launches",
]
