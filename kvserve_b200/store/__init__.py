"""Shared KV store for prefix reuse across requests and engines on one node
(role of the reference's MooncakeStoreConnector,
kvsfuse-vllm0.30.0/mooncake/store/*.py).  Blocks are keyed by chained
prefix hashes; values live in a tiered pool (GPU HBM, pinned host memory,
disk) with LRU demotion; values may be stored compressed with any profile of
the modular pipeline (the reference stores raw blocks only)."""
from .hashing import block_hashes, chunk_hashes
from .layout import PoolKey, RankLocalLayout, TPShardedLayout
from .pool import TieredKVPool
from .connector import KVStoreConnector

__all__ = ["block_hashes", "chunk_hashes", "PoolKey", "RankLocalLayout", "TPShardedLayout", "TieredKVPool",
           "KVStoreConnector"]
