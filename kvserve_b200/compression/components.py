"""Component interfaces of the modular pipeline
``Raw KV -> Transformer -> Quantizer -> Codec -> Compressed KV``
(kvserve_v1/compression/components.py:11-109).

KV tensors handed to a stage are one layer ``[2, num_blocks, block_size,
num_kv_heads, head_size]`` (transformer / quantizer) or the stacked codec
buffer (codec).  Every concrete component also accepts ``update_params`` so
one instance can follow per-request configuration changes.
"""
from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Any

import torch


class Transformer(ABC):
    """Invertible per-layer transform of KV values."""

    @abstractmethod
    def transform(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any) -> torch.Tensor:
        ...

    @abstractmethod
    def inverse(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any) -> torch.Tensor:
        ...

    def update_params(self, **kwargs: Any) -> None:  # pragma: no cover - default no-op
        pass


class Quantizer(ABC):
    """Lossy map of one layer's KV to uint8 symbols plus parameters."""

    @abstractmethod
    def quantize(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any) -> tuple[torch.Tensor, dict]:
        ...

    @abstractmethod
    def dequantize(self, layer_id: int, tensor: torch.Tensor, meta: Any, **kwargs: Any) -> torch.Tensor:
        ...

    def update_params(self, **kwargs: Any) -> None:  # pragma: no cover
        pass


class Codec(ABC):
    """Lossless coding of the stacked symbol (or raw byte) buffer."""

    @abstractmethod
    def encode(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any) -> torch.Tensor:
        ...

    @abstractmethod
    def decode(self, layer_id: int, tensor: torch.Tensor, original_dtype: str, original_shape: list,
               device: str, **kwargs: Any) -> torch.Tensor:
        ...

    def update_params(self, **kwargs: Any) -> None:  # pragma: no cover
        pass
