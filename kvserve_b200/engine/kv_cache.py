"""Paged KV cache of the decode engine.

One tensor ``[L, 2, num_blocks, block_size, Hkv, D]`` (the NHD block layout
the reference forces on vLLM, kvserve_v1/connector/compressed_kv_connector.py:216-231)
plus a free-list block allocator.  Block tables are int32 device tensors.
"""
from __future__ import annotations

from typing import Optional

import torch


class PagedKVCache:
    def __init__(self, num_layers: int, num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int,
                 device, dtype=torch.bfloat16):
        self.num_layers, self.num_blocks, self.block_size = num_layers, num_blocks, block_size
        self.num_kv_heads, self.head_dim = num_kv_heads, head_dim
        self.cache = torch.zeros((num_layers, 2, num_blocks, block_size, num_kv_heads, head_dim), dtype=dtype,
                                 device=device)
        self._free = list(range(num_blocks - 1, -1, -1))

    @property
    def bytes(self) -> int:
        return self.cache.numel() * self.cache.element_size()

    def blocks_for(self, num_tokens: int) -> int:
        return (num_tokens + self.block_size - 1) // self.block_size

    def num_free(self) -> int:
        return len(self._free)

    def allocate(self, num_tokens: int) -> list[int]:
        n = self.blocks_for(num_tokens)
        if n > len(self._free):
            raise MemoryError(f"KV cache exhausted: need {n} blocks, {len(self._free)} free")
        return [self._free.pop() for _ in range(n)]

    def extend(self, blocks: list[int], num_tokens: int) -> list[int]:
        need = self.blocks_for(num_tokens) - len(blocks)
        if need > 0:
            blocks = blocks + self.allocate(need * self.block_size)
        return blocks

    def release(self, blocks: list[int]) -> None:
        self._free.extend(reversed(blocks))

    def block_table(self, blocks: list[int], width: Optional[int] = None) -> torch.Tensor:
        width = width or len(blocks)
        t = torch.zeros(width, dtype=torch.int32)
        t[: len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
        return t.to(self.cache.device, non_blocking=True)

    def slot(self, blocks: list[int], position: int) -> int:
        return blocks[position // self.block_size] * self.block_size + position % self.block_size
