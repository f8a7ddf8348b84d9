"""KV-cache group rules shared by the connectors.

vLLM describes a model's paged KV cache as one or more groups, each with a
spec (full attention, sliding window, ...).  The connectors of this package
move one group; a sliding-window group keeps real blocks only for the last
window of tokens (older ones become vLLM's null block), which limits what can
be sent or stored.
"""
from __future__ import annotations


def sliding_window_blocks(kv_cache_config, connector: str = "this connector") -> int:
    """How many trailing blocks of a request carry KV that attention still
    reads, for a sliding-window group (0: full attention, every block).  vLLM
    swaps blocks that fell out of the window for its null block, so only the
    last ``ceil(window / block_size) + 1`` hold KV (the window's first token
    may sit inside a block, which adds one).  The role of the reference's
    sliding-window clip, kvsfuse-vllm0.30.0/mooncake/mooncake_connector.py:833-862.
    A hybrid layout with several groups is refused rather than half-moved."""
    groups = list(getattr(kv_cache_config, "kv_cache_groups", None) or [])
    if len(groups) > 1:
        raise ValueError(f"{connector} transfers one KV-cache group, this model has {len(groups)}; "
                         "run vLLM with the hybrid KV-cache manager disabled")
    if not groups:
        return 0
    spec = getattr(groups[0], "kv_cache_spec", None)
    window = getattr(spec, "sliding_window", None)
    # a FullAttentionSpec may carry a window too (hybrid manager off): then
    # every block stays allocated, and possibly prefix-cached, so all move
    if type(spec).__name__ != "SlidingWindowSpec" or not window:
        return 0
    return -(-int(window) // int(spec.block_size)) + 1
