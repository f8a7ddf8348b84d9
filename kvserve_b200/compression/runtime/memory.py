"""Memory plan of the fixed-profile runtime (role of
kvserve_v1/compression/runtime/memory.py:233-403): everything the runtime
will allocate is computed up front, from the geometry alone, so the caller
can reserve it before sizing its inference KV cache.

Per slot: an arena of one frame per layer (``frame_stride`` bytes each, the
largest frame of a chunk), the lossless-codec output bank and its scratch.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from ...ops.kv_codec import FrameSpec, RAW_BITS, bits_for_levels, frame_layout
from .config import CompressionConfig
from .scores import HeadSelection, build_head_selection
from .spec import CacheSpec, round_up

ALIGNMENT = 256
METADATA_BYTES = 1 << 20
GUARD_BYTES = 4 << 20
RZE_CHUNK = 16384


@dataclass(frozen=True)
class LayerEntry:
    name: str
    layer_index: int
    dense_index: int
    group: int
    heads: int
    head_size: int
    n_low: int


@dataclass(frozen=True)
class RuntimeLayout:
    layers: tuple
    block_size: int
    chunk_tokens: int
    frame_stride: int
    arena_bytes: int
    codec_capacity: int
    codec_scratch: int

    def spec(self, config: CompressionConfig, entry: LayerEntry, part: int, tokens: int) -> FrameSpec:
        return frame_spec(config, entry, part, tokens)


def frame_spec(config: CompressionConfig, e: LayerEntry, part: int, tokens: int) -> FrameSpec:
    """Frame of one (layer, part): the other part's sections are empty-raw so
    the frame only carries what this part needs."""
    H, D = e.heads, e.head_size
    if not config.uses_quantizer:
        return FrameSpec(tokens, H, D, e.n_low, ((RAW_BITS, RAW_BITS), (RAW_BITS, RAW_BITS)), ((2, 2), (2, 2)),
                         transform=False)
    kl = (config.low_key_num_levels, config.high_key_num_levels)
    vl = (config.low_value_num_levels, config.high_value_num_levels)
    bits = ((bits_for_levels(kl[0]), bits_for_levels(kl[1])), (bits_for_levels(vl[0]), bits_for_levels(vl[1])))
    return FrameSpec(tokens, H, D, e.n_low, bits, (kl, vl), transform=config.uses_transformer)


def _rze_max(n: int) -> int:
    chunks = (n + RZE_CHUNK - 1) // RZE_CHUNK
    return 24 + 4 * chunks + chunks * (RZE_CHUNK // 16 + RZE_CHUNK + 16 + 4)


def _rze_scratch(n: int) -> int:
    chunks = (n + RZE_CHUNK - 1) // RZE_CHUNK
    return chunks * (RZE_CHUNK // 16 + RZE_CHUNK + 16 + 4 + 8) + 16


@dataclass
class CompressionMemoryPlan:
    config: CompressionConfig
    specs: dict
    layout: RuntimeLayout
    selection: HeadSelection
    blocks_per_logical: int
    tp_rank: int
    tp_size: int
    num_layers: int
    slot_bytes: int
    reserved_bytes: int
    output_slot_bytes: int = 0
    device: Optional[torch.device] = None


def build_memory_plan(config: CompressionConfig, specs: dict[str, CacheSpec], blocks_per_logical: int = 1,
                      tp_size: int = 1, tp_rank: int = 0, num_layers: Optional[int] = None, device=None,
                      scores: Optional[np.ndarray] = None, group_indices: Optional[dict] = None) -> CompressionMemoryPlan:
    if not specs:
        raise ValueError("the runtime needs at least one cache spec")
    items = sorted(specs.items(), key=lambda kv: kv[1].layer_index)
    if len({s.block_size for _, s in items}) != 1:
        raise ValueError("the runtime requires a common block size")
    for name, s in items:
        if s.dtype is not torch.bfloat16:
            raise ValueError(f"the runtime supports bf16 KV caches only (layer {name} is {s.dtype})")
        if s.head_size != s.head_size_v:
            raise ValueError("the fused frame path needs equal K and V head sizes")
        if s.head_size not in (64, 128, 256) or s.num_kv_heads * s.head_size > 2048:
            raise ValueError("the fused frame path supports head_size 64/128/256 and H*D <= 2048 per rank")
    L = num_layers if num_layers is not None else (max(s.layer_index for _, s in items) + 1)
    if config.enabled and config.uses_quantizer and config.split_type == "head":
        sel = build_head_selection(dict(items), config, tp_rank, tp_size, scores)
    else:
        sel = HeadSelection({s.layer_index: 0 for _, s in items},
                            {s.layer_index: tuple(range(s.num_kv_heads)) for _, s in items})
    group_indices = group_indices or {}
    entries = []
    for d, (name, s) in enumerate(items):
        if config.split_type == "layer" and config.uses_quantizer:
            low_layers = round(L * 0.33)
            n_low = s.num_kv_heads if low_layers > 0 and s.layer_index >= L - low_layers else 0
        else:
            n_low = sel.low_counts.get(s.layer_index, 0)
        entries.append(LayerEntry(name, s.layer_index, d, group_indices.get(name, 0), s.num_kv_heads, s.head_size,
                                  n_low))
    bs = items[0][1].block_size
    chunk_tokens = config.logical_blocks_per_chunk * blocks_per_logical * bs
    stride = 0
    for e in entries:
        for part in (0, 1):
            stride = max(stride, frame_layout(frame_spec(config, e, part, chunk_tokens)).frame_bytes)
    stride = round_up(stride, ALIGNMENT)
    arena = stride * len(entries)
    cap = _rze_max(arena) if config.uses_codec else 0
    scr = _rze_scratch(arena) if config.uses_codec else 0
    layout = RuntimeLayout(tuple(entries), bs, chunk_tokens, stride, arena, round_up(cap, ALIGNMENT),
                           round_up(scr, ALIGNMENT))
    slot_bytes = layout.arena_bytes + layout.codec_capacity + layout.codec_scratch
    reserved = config.slot_count * slot_bytes + METADATA_BYTES + GUARD_BYTES
    return CompressionMemoryPlan(config, dict(items), layout, sel, blocks_per_logical, tp_rank, tp_size, L, slot_bytes,
                                 reserved, device=torch.device(device) if device is not None else None)
