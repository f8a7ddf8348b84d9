"""Decoder model shapes used by the engine and the benchmarks (random-init
weights of these architectures; no checkpoints are needed)."""
from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Optional


@dataclass(frozen=True)
class ModelConfig:
    name: str
    num_layers: int
    hidden: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5
    qkv_bias: bool = False
    max_position: int = 131072
    score_model_name: Optional[str] = None  # head-score table to use

    @property
    def q_size(self) -> int:
        return self.num_q_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        return 2 * self.num_layers * self.kv_size * dtype_bytes

    def params(self) -> int:
        per_layer = (self.hidden * (self.q_size + 2 * self.kv_size) + self.q_size * self.hidden
                     + 3 * self.hidden * self.intermediate + 2 * self.hidden)
        return self.num_layers * per_layer + 2 * self.vocab * self.hidden + self.hidden

    def with_layers(self, n: int) -> "ModelConfig":
        return replace(self, num_layers=n)


PRESETS: dict[str, ModelConfig] = {
    "llama-3.1-8b": ModelConfig("llama-3.1-8b", 32, 4096, 32, 8, 128, 14336, 128256, 500000.0,
                                score_model_name="Llama-3.1-8B-Instruct"),
    "qwen2.5-7b": ModelConfig("qwen2.5-7b", 28, 3584, 28, 4, 128, 18944, 152064, 1000000.0, 1e-6, qkv_bias=True,
                              score_model_name="Qwen2.5-7B-Instruct"),
    "llama-3-70b": ModelConfig("llama-3-70b", 80, 8192, 64, 8, 128, 28672, 128256, 500000.0),
    "qwen2.5-32b": ModelConfig("qwen2.5-32b", 64, 5120, 40, 8, 128, 27648, 152064, 1000000.0, 1e-6, qkv_bias=True,
                               score_model_name="Qwen2.5-32B-Instruct"),
    # small shapes for tests and smoke runs
    "tiny": ModelConfig("tiny", 2, 512, 8, 2, 128, 1024, 1024, 10000.0),
    "tiny-gqa": ModelConfig("tiny-gqa", 4, 1024, 16, 4, 128, 2048, 4096, 500000.0),
}


def get_config(name: str) -> ModelConfig:
    key = name.lower()
    if key not in PRESETS:
        raise KeyError(f"unknown model {name!r}; presets: {sorted(PRESETS)}")
    return PRESETS[key]
