"""Block-indexed gather/scatter of one request's KV from/to a paged cache
(behaviour of kvserve_v1/utils/kv_utils.py).

Two paged layouts are recognised by where the K/V axis of size 2 sits:
FlashAttention ``[2, num_blocks, block_size, ...]`` and MLA/FlashInfer
``[num_blocks, 2, block_size, ...]``.  The gathered tensor keeps the layout
of the cache (``[2, nb, bs, H, D]`` resp. ``[nb, 2, bs, H, D]``).
"""
from __future__ import annotations

import torch


def make_slot_mapping(token_ids: list, block_ids: list, block_size: int) -> torch.Tensor:
    """Absolute cache slots of a request's tokens (CPU int64 [num_tokens])."""
    b = torch.tensor(block_ids, dtype=torch.long)
    slots = (b[:, None] * block_size + torch.arange(block_size, dtype=torch.long)[None]).flatten()
    return slots[: len(token_ids)]


def _kv_axis(kv: torch.Tensor) -> int:
    if kv.shape[0] == 2:
        return 0
    if kv.dim() > 1 and kv.shape[1] == 2:
        return 1
    raise RuntimeError(f"Unsupported KV layout shape: {tuple(kv.shape)}")


def extract_kv_from_layer(kv_layer: torch.Tensor, slot_mapping: torch.Tensor) -> torch.Tensor:
    """[2, num_pages, page_size, ...] -> [2, num_tokens, kv_dim]."""
    flat = kv_layer.reshape(2, kv_layer.shape[1] * kv_layer.shape[2], -1)
    return flat[:, slot_mapping.to(flat.device), :].clone()


def inject_kv_into_layer(kv_cache_layer: torch.Tensor, kv_data: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    flat = kv_cache_layer.reshape(2, kv_cache_layer.shape[1] * kv_cache_layer.shape[2], -1)
    flat[:, slot_mapping.to(flat.device), :] = kv_data.to(flat.device)


def extract_kv_from_layer_by_blocks(kv_layer: torch.Tensor, block_ids: list) -> torch.Tensor:
    ax = _kv_axis(kv_layer)
    if not block_ids:
        return (kv_layer[:, :0] if ax == 0 else kv_layer[:0]).clone()
    idx = torch.tensor(block_ids, device=kv_layer.device, dtype=torch.long)
    return kv_layer[:, idx].clone() if ax == 0 else kv_layer[idx].clone()


def inject_kv_into_layer_by_blocks(kv_cache_layer: torch.Tensor, kv_data: torch.Tensor, block_ids: list,
                                   request_id: str = "") -> None:
    """Scatter a request's blocks back; when producer and consumer block counts
    differ only in tail blocks, the overlapping blocks are written."""
    if not block_ids:
        return
    ax = _kv_axis(kv_cache_layer)
    idx = torch.tensor(block_ids, device=kv_cache_layer.device, dtype=torch.long)
    data = kv_data.to(kv_cache_layer.device)
    n = data.shape[1] if ax == 0 else data.shape[0]
    idx = idx[:n]
    if ax == 0:
        kv_cache_layer[:, idx] = data[:, : idx.numel()]
    else:
        kv_cache_layer[idx] = data[: idx.numel()]
