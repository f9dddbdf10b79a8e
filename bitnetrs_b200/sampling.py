"""Sampling hyper-parameters of the generate API: SamplingConfig
(crates/bitnet-inference/src/lib.rs:80-178) with the reference's presets and
validation rules.  The device sampler (bitnet_cuda_sample_next_token,
CudaBackend.sample_next_token, BitNetModel.generate(sampling=...)) runs the
reference's sample_next_token on the GPU; greedy decode (top_k == 1) also
runs as an argmax fused after the lm_head.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

from .errors import InvalidConfig


@dataclass(frozen=True)
class SamplingConfig:
    temperature: float = 0.7
    top_p: float = 0.9
    top_k: int = 50
    repetition_penalty: float = 1.1
    max_new_tokens: int = 512
    seed: int = 0

    @staticmethod
    def greedy() -> "SamplingConfig":
        """SamplingConfig::greedy (lib.rs:115-124)."""
        return SamplingConfig(1.0, 1.0, 1, 1.0, 256, 42)

    @staticmethod
    def chat_defaults() -> "SamplingConfig":
        """SamplingConfig::chat_defaults (lib.rs:127-136); also the Default."""
        return SamplingConfig(0.7, 0.9, 50, 1.1, 512, 0)

    @staticmethod
    def creative() -> "SamplingConfig":
        """SamplingConfig::creative (lib.rs:139-148)."""
        return SamplingConfig(1.0, 0.95, 0, 1.05, 1024, 0)

    def is_greedy(self) -> bool:
        """sample_next_token's greedy shortcut (lib.rs:262-270) applies: the
        argmax of the (penalised, tempered) logits."""
        return self.top_k == 1

    def to_c(self):
        from ._native import Sampling

        return Sampling(self.temperature, self.top_p, self.top_k, self.repetition_penalty, self.seed)

    def with_(self, **kw) -> "SamplingConfig":
        return replace(self, **kw)

    def validate(self) -> None:
        """SamplingConfig::validate (lib.rs:160-178), same checks and order."""
        if not self.temperature > 0.0:
            raise InvalidConfig(f"temperature must be > 0, got {self.temperature}")
        if not 0.0 < self.top_p <= 1.0:
            raise InvalidConfig(f"top_p must be in (0, 1], got {self.top_p}")
        if self.repetition_penalty < 1.0:
            raise InvalidConfig(f"repetition_penalty must be >= 1.0, got {self.repetition_penalty}")
        if self.max_new_tokens == 0:
            raise InvalidConfig("max_new_tokens must be > 0")
