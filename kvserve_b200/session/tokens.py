"""Token accounting of a session (role of
kvsfuse-vllm0.30.0/mooncake/compression/tokens.py:6-34).  The decode side
may already hold a block-aligned prefix of the prompt; only the suffix is
transferred, chunk by chunk."""
from __future__ import annotations


def suffix_token_counts(num_tokens: int, block_ids: list, block_sizes: dict) -> dict:
    """Valid tokens per KV-cache group in the transferred suffix: the prompt
    covers ``ceil(num_tokens / bs)`` blocks, the consumer sent block ids only
    for the suffix it lacks, so the suffix starts ``(full - sent) * bs``
    tokens in.  A group with no block ids (full prefix hit or release-only
    notification) transfers nothing."""
    out = {}
    for group, bs in block_sizes.items():
        full = -(-num_tokens // bs)
        sent = len(block_ids[group]) if block_ids else 0
        out[group] = num_tokens - (full - sent) * bs if sent else 0
    return out


def chunk_token_counts(valid_tokens_by_group: dict, block_sizes: dict, logical_start: int,
                       logical_count: int) -> dict:
    """Tokens of each group inside logical blocks ``[start, start + count)``
    of the suffix."""
    out = {}
    for group, bs in block_sizes.items():
        remaining = valid_tokens_by_group[group] - logical_start * bs
        out[group] = max(0, min(remaining, logical_count * bs))
    return out
