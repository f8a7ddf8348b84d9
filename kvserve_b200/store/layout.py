"""Store key layouts.  A key names one chunk of one model's KV for one shard:

* :class:`RankLocalLayout` — every TP rank stores and reads its own shard
  (``tp{rank}of{size}``); engines with the same TP size share entries.
* :class:`TPShardedLayout` — shards are keyed by KV-head range, so an engine
  with another TP size can still find the heads it owns (as long as its
  head ranges are unions of stored ones).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class PoolKey:
    model: str
    shard: str
    chunk_hash: bytes

    def to_string(self) -> str:
        return f"{self.model}/{self.shard}/{self.chunk_hash.hex()}"


class RankLocalLayout:
    def __init__(self, model: str, tp_rank: int, tp_size: int):
        self.model, self.tp_rank, self.tp_size = model, tp_rank, tp_size

    def shards(self) -> list[str]:
        return [f"tp{self.tp_rank}of{self.tp_size}"]

    def key(self, shard: str, chunk_hash: bytes) -> PoolKey:
        return PoolKey(self.model, shard, chunk_hash)


class TPShardedLayout:
    def __init__(self, model: str, tp_rank: int, tp_size: int, num_kv_heads: int, store_tp_size: int):
        if num_kv_heads % store_tp_size or num_kv_heads % tp_size:
            raise ValueError("KV heads must divide both TP sizes")
        self.model = model
        lo = tp_rank * num_kv_heads // tp_size
        hi = (tp_rank + 1) * num_kv_heads // tp_size
        step = num_kv_heads // store_tp_size
        self.ranges = [(h, h + step) for h in range(0, num_kv_heads, step) if lo <= h and h + step <= hi]
        if not self.ranges:
            raise ValueError("this rank's heads are not a union of stored shards (store TP size too small)")

    def shards(self) -> list[str]:
        return [f"heads{a}-{b}" for a, b in self.ranges]

    def key(self, shard: str, chunk_hash: bytes) -> PoolKey:
        return PoolKey(self.model, shard, chunk_hash)
