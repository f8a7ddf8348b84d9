"""Prefix-reuse connector over the tiered pool (role of
kvsfuse-vllm0.30.0/mooncake/store/connector.py:125-411 and worker.py).

The paged KV of a request ``[L, 2, blocks, block_size, H, D]`` is stored per
chunk of ``blocks_per_chunk`` blocks under its chained prefix hash;
``lookup`` returns how many leading tokens are available, ``load`` copies
them into the caller's paged blocks.  With ``compression`` (any profile of
the modular pipeline) values are stored compressed and restored on load.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from .hashing import block_hashes, chunk_hashes
from .layout import RankLocalLayout
from .pool import TieredKVPool


class KVStoreConnector:
    def __init__(self, pool: TieredKVPool, block_size: int, blocks_per_chunk: int = 16, layout=None,
                 compression: Optional[dict] = None, num_kv_heads: int = 0, head_size: int = 0,
                 num_layers: Optional[int] = None, salt: bytes = b""):
        self.pool, self.block_size, self.bpc = pool, block_size, blocks_per_chunk
        self.layout = layout or RankLocalLayout("model", 0, 1)
        self.salt = salt
        self.adapter = None
        if compression is not None:
            from ..compression.adapter import KVCompressionAdapter
            self.adapter = KVCompressionAdapter(compression, num_kv_heads, head_size, num_layers=num_layers)

    @property
    def chunk_tokens(self) -> int:
        return self.block_size * self.bpc

    def _keys(self, token_ids: Sequence[int]) -> list[str]:
        ch = chunk_hashes(block_hashes(token_ids, self.block_size, extra=self.salt), self.bpc)
        shard = self.layout.shards()[0]
        return [self.layout.key(shard, h).to_string() for h in ch]

    def lookup(self, token_ids: Sequence[int]) -> int:
        """Tokens of the longest stored prefix (a multiple of the chunk size)."""
        n = 0
        for key in self._keys(token_ids):
            if not self.pool.contains(key):
                break
            n += 1
        return n * self.chunk_tokens

    def save(self, token_ids: Sequence[int], kv: torch.Tensor, block_ids: Sequence[int]) -> int:
        """Store every full chunk of the request's KV (``kv`` is the paged
        cache ``[L, 2, num_blocks, block_size, H, D]``); returns chunks written."""
        written = 0
        for c, key in enumerate(self._keys(token_ids)):
            if self.pool.contains(key):
                continue
            ids = torch.tensor(block_ids[c * self.bpc:(c + 1) * self.bpc], device=kv.device, dtype=torch.long)
            value = kv.index_select(2, ids)
            if self.adapter is not None:
                value = self.adapter.compress(value, key) or value
            self.pool.put(key, value)
            written += 1
        return written

    def load(self, token_ids: Sequence[int], kv: torch.Tensor, block_ids: Sequence[int],
             num_tokens: Optional[int] = None) -> int:
        """Copy the stored prefix into ``kv``'s blocks; returns tokens loaded."""
        limit = self.lookup(token_ids) if num_tokens is None else num_tokens
        loaded = 0
        for c, key in enumerate(self._keys(token_ids)):
            if loaded >= limit:
                break
            value = self.pool.get(key)
            if value is None:
                break
            if not isinstance(value, torch.Tensor):
                value = self.adapter.decompress(value)
            ids = torch.tensor(block_ids[c * self.bpc:(c + 1) * self.bpc], device=kv.device, dtype=torch.long)
            kv.index_copy_(2, ids, value.to(kv.device, kv.dtype))
            loaded += self.chunk_tokens
        return loaded
