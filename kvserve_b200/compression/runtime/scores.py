"""Head selection of the fixed-profile runtime (semantics of
kvserve_v1/compression/runtime/scores.py:45-112): a stable global argsort of
the scores of the layers present picks ``round(n * hybrid_ratio)`` low heads;
per layer the local order is low heads first, both groups ascending; TP ranks
slice columns, and ranks that replicate a KV head (``tp_size > kv_heads``)
map to head ``tp_rank // (tp_size // kv_heads)``."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

from ..heads import load_scores_file
from .config import CompressionConfig
from .spec import CacheSpec


@dataclass(frozen=True)
class HeadSelection:
    low_counts: dict
    local_orders: dict


def build_head_selection(specs: dict[str, CacheSpec], config: CompressionConfig, tp_rank: int, tp_size: int,
                         scores: Optional[np.ndarray] = None) -> HeadSelection:
    items = list(specs.items())
    if config.split_type == "layer":
        return HeadSelection({s.layer_index: 0 for _, s in items},
                             {s.layer_index: tuple(range(s.num_kv_heads)) for _, s in items})
    if scores is None:
        if not config.score_path:
            raise ValueError("Head split requires a score_path or head scores.")
        scores = load_scores_file(config.score_path).numpy()
    scores = np.asarray(scores, dtype=np.float32)
    if scores.ndim != 2 or not np.isfinite(scores).all():
        raise ValueError("Head scores must be a finite 2D array of layers and KV heads.")
    cand = []
    for _, s in items:
        if not 0 <= s.layer_index < scores.shape[0]:
            raise ValueError(f"Head scores have no row for layer {s.layer_index}.")
        base = s.layer_index * scores.shape[1]
        cand.extend(range(base, base + scores.shape[1]))
    cand = np.asarray(cand, dtype=np.int64)
    mask = np.zeros(scores.size, dtype=bool)
    n_low = round(cand.size * config.hybrid_ratio)
    if n_low:
        sel = np.argsort(scores.reshape(-1)[cand], kind="stable")[:n_low]
        mask[cand[sel]] = True
    mask = mask.reshape(scores.shape)
    low_counts, orders = {}, {}
    for _, s in items:
        H, W = s.num_kv_heads, mask.shape[1]
        if W == H:
            start = 0
        elif W == H * tp_size:
            start = tp_rank * H
        elif H == 1 and 0 < W < tp_size and tp_size % W == 0:
            start = tp_rank // (tp_size // W)
        else:
            raise ValueError(f"Head score width {W} is incompatible with {H} local KV heads and TP size {tp_size}.")
        local = mask[s.layer_index, start:start + H]
        low = np.flatnonzero(local).tolist()
        high = np.flatnonzero(~local).tolist()
        low_counts[s.layer_index] = len(low)
        orders[s.layer_index] = tuple(low + high)
    return HeadSelection(low_counts, orders)
