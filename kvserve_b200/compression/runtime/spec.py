"""Per-layer cache geometry accepted by the runtime (vLLM-independent)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch


def round_up(value: int, alignment: int) -> int:
    return (value + alignment - 1) // alignment * alignment


@dataclass(frozen=True)
class CacheSpec:
    layer_index: int
    block_size: int
    num_kv_heads: int
    head_size: int
    dtype: torch.dtype
    head_size_v: Optional[int] = None

    def __post_init__(self):
        if self.head_size_v is None:
            object.__setattr__(self, "head_size_v", self.head_size)
