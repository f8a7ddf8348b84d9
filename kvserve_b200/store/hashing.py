"""Chained prefix hashes of token blocks: the hash of block i covers every
token up to the end of block i, so equal hashes mean equal prefixes."""
from __future__ import annotations

import hashlib
from typing import Optional, Sequence

import numpy as np

ROOT = b"kvserve-b200-prefix-root"


def block_hashes(token_ids: Sequence[int], block_size: int, parent: Optional[bytes] = None,
                 extra: bytes = b"") -> list[bytes]:
    """Hashes of the full blocks of ``token_ids`` (a trailing partial block
    has none).  ``extra`` salts the chain (e.g. a model or LoRA identity)."""
    h = parent if parent is not None else hashlib.blake2b(ROOT + extra, digest_size=16).digest()
    arr = np.asarray(token_ids, dtype=np.int64)
    out = []
    for b in range(len(arr) // block_size):
        h = hashlib.blake2b(h + arr[b * block_size:(b + 1) * block_size].tobytes(), digest_size=16).digest()
        out.append(h)
    return out


def chunk_hashes(hashes: Sequence[bytes], blocks_per_chunk: int) -> list[bytes]:
    """Every ``blocks_per_chunk``-th block hash: the key of each full chunk."""
    return [hashes[i] for i in range(blocks_per_chunk - 1, len(hashes), blocks_per_chunk)]
