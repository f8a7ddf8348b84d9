"""Prefix-reuse connector over the tiered pool (role of
kvsfuse-vllm0.30.0/mooncake/store/connector.py:125-411 and worker.py).

The paged KV of a request is stored per chunk of ``blocks_per_chunk``
blocks under its chained prefix hash, as one ``[L, 2, blocks, block_size, H,
D]`` value; ``lookup`` returns how many leading tokens are available,
``load`` copies them into the caller's paged blocks.  The caller's cache is
either one stacked tensor ``[L, 2, num_blocks, block_size, H, D]`` or a list
of per-layer caches in vLLM's layouts (``[2, num_blocks, ...]`` or
``[num_blocks, 2, ...]``).  With ``compression`` (any profile of the modular
pipeline) values are stored compressed, in the wire form of
:mod:`kvserve_b200.compression.wire` (tensors and plain metadata, so they
can live in files), and restored on load.
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

    @staticmethod
    def _gather(kv, ids: torch.Tensor) -> torch.Tensor:
        """``[L, 2, len(ids), block_size, H, D]`` of the given blocks."""
        if isinstance(kv, torch.Tensor):
            return kv.index_select(2, ids)
        return torch.stack([t.index_select(1, ids) if t.shape[0] == 2 else t.index_select(0, ids).transpose(0, 1)
                            for t in kv])

    @staticmethod
    def _scatter(kv, ids: torch.Tensor, value: torch.Tensor) -> None:
        if isinstance(kv, torch.Tensor):
            kv.index_copy_(2, ids, value.to(kv.device, kv.dtype))
            return
        for t, v in zip(kv, value):
            v = v.to(t.device, t.dtype)
            if t.shape[0] == 2:
                t.index_copy_(1, ids, v)
            else:
                t.index_copy_(0, ids, v.transpose(0, 1))

    def _encode(self, value: torch.Tensor, key: str):
        if self.adapter is None:
            return value
        c = self.adapter.compress(value, key)
        if c is None:
            return value
        from ..compression.wire import build_wire
        w = build_wire(c, 1 << 62)
        return {"meta": w.meta, "body": list(w.body_chunks), "aux": list(w.aux_tensors)}

    def _decode(self, stored) -> torch.Tensor:
        if isinstance(stored, torch.Tensor):
            return stored
        from ..compression.wire import CompressedWire, restore_from_wire
        return self.adapter.decompress(restore_from_wire(CompressedWire(stored["meta"], stored["body"],
                                                                        stored["aux"])))

    def save(self, token_ids: Sequence[int], kv, block_ids: Sequence[int]) -> int:
        """Store every full chunk of the request's KV (``kv``: the stacked
        paged cache or the list of per-layer caches); returns chunks written."""
        written = 0
        dev = kv.device if isinstance(kv, torch.Tensor) else kv[0].device
        for c, key in enumerate(self._keys(token_ids)):
            if self.pool.contains(key):
                continue
            ids = torch.tensor(block_ids[c * self.bpc:(c + 1) * self.bpc], device=dev, dtype=torch.long)
            self.pool.put(key, self._encode(self._gather(kv, ids), key))
            written += 1
        return written

    def load(self, token_ids: Sequence[int], kv, block_ids: Sequence[int],
             num_tokens: Optional[int] = None, first_block: int = 0) -> int:
        """Copy the stored prefix into the cache's blocks, skipping the first
        ``first_block`` blocks (already present, e.g. a local prefix-cache
        hit); returns the tokens of the prefix that are now in place (chunk
        granularity, counted from token 0)."""
        limit = self.lookup(token_ids) if num_tokens is None else num_tokens
        dev = kv.device if isinstance(kv, torch.Tensor) else kv[0].device
        loaded = 0
        for c, key in enumerate(self._keys(token_ids)):
            if loaded >= limit:
                break
            lo, hi = c * self.bpc, (c + 1) * self.bpc
            if hi <= first_block:                 # wholly present already
                loaded += self.chunk_tokens
                continue
            stored = self.pool.get(key)
            if stored is None:
                break
            value = self._decode(stored)
            skip = max(0, first_block - lo)
            ids = torch.tensor(block_ids[lo + skip:hi], device=dev, dtype=torch.long)
            self._scatter(kv, ids, value[:, :, skip:])
            loaded += self.chunk_tokens
        return loaded
