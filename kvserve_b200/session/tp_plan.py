"""KV transfer planning between producer and consumer groups of different
tensor-parallel sizes (roles of
kvsfuse-vllm0.30.0/mooncake/mooncake_connector.py:243-447 — TP ratio, per-pair
copy plan with replicated KV heads, region-length validation — and
kvsfuse-vllm0.30.0/mooncake/session_ipc.py:34-41, the ranks a rank pairs with).

Formulated over KV-head ranges.  A TP rank holds a contiguous range of the
model's KV heads (``num_kv_heads / tp`` of them) or, when the TP size exceeds
the head count, one replicated head.  The plan gives every consumer rank each
of its heads exactly once, from a producer rank that holds it; among the
replicas of a head the producer ``consumer_rank % replicas`` is used, which
spreads the senders.  Copies of consecutive heads between the same two ranks
are merged, so homogeneous TP is one full-shard copy per pair, TP p -> 1 is p
copies into disjoint head offsets of the consumer's block, and TP 1 -> c is c
disjoint slices of the producer's block.  Byte offsets follow from the
per-head length of a block (``block_size * head_dim * dtype bytes`` for NHD
K or V halves).
"""
from __future__ import annotations

from dataclasses import dataclass


def tp_ratio(local_tp: int, remote_tp: int) -> int:
    """``local/remote`` when local >= remote, else ``-(remote/local)``; the
    larger size must be a multiple of the smaller."""
    if local_tp < 1 or remote_tp < 1:
        raise ValueError("TP sizes must be positive")
    if local_tp >= remote_tp:
        if local_tp % remote_tp:
            raise ValueError(f"local TP {local_tp} is not a multiple of remote TP {remote_tp}")
        return local_tp // remote_tp
    if remote_tp % local_tp:
        raise ValueError(f"remote TP {remote_tp} is not a multiple of local TP {local_tp}")
    return -(remote_tp // local_tp)


@dataclass(frozen=True)
class HeadShard:
    first: int      # first global KV head held
    count: int      # number of heads held
    replica: int    # replica index of this shard (0 when heads are not replicated)
    replicas: int   # ranks holding the same heads


def head_shard(tp_rank: int, tp_size: int, num_kv_heads: int) -> HeadShard:
    if not 0 <= tp_rank < tp_size:
        raise ValueError("tp_rank out of range")
    if tp_size <= num_kv_heads:
        if num_kv_heads % tp_size:
            raise ValueError(f"{num_kv_heads} KV heads do not split over TP {tp_size}")
        n = num_kv_heads // tp_size
        return HeadShard(tp_rank * n, n, 0, 1)
    if tp_size % num_kv_heads:
        raise ValueError(f"TP {tp_size} does not replicate {num_kv_heads} KV heads evenly")
    reps = tp_size // num_kv_heads
    return HeadShard(tp_rank // reps, 1, tp_rank % reps, reps)


@dataclass(frozen=True)
class HeadCopy:
    src_rank: int
    dst_rank: int
    src_head: int   # first head, local index in the producer's shard
    dst_head: int   # first head, local index in the consumer's shard
    heads: int

    def byte_range(self, bytes_per_head: int) -> tuple[int, int, int]:
        """(source offset, destination offset, length) inside one block's
        K or V half of ``heads * bytes_per_head`` bytes per rank."""
        return self.src_head * bytes_per_head, self.dst_head * bytes_per_head, self.heads * bytes_per_head


def transfer_plan(producer_tp: int, consumer_tp: int, num_kv_heads: int) -> list[HeadCopy]:
    shards_p = [head_shard(r, producer_tp, num_kv_heads) for r in range(producer_tp)]
    plan: list[HeadCopy] = []
    for d in range(consumer_tp):
        ds = head_shard(d, consumer_tp, num_kv_heads)
        for h in range(ds.first, ds.first + ds.count):
            holders = [p for p, s in enumerate(shards_p) if s.first <= h < s.first + s.count]
            src = holders[d % len(holders)]
            sh = h - shards_p[src].first
            dh = h - ds.first
            last = plan[-1] if plan else None
            if (last is not None and last.src_rank == src and last.dst_rank == d
                    and last.src_head + last.heads == sh and last.dst_head + last.heads == dh):
                plan[-1] = HeadCopy(src, d, last.src_head, last.dst_head, last.heads + 1)
            else:
                plan.append(HeadCopy(src, d, sh, dh, 1))
    return plan


def target_ranks(producer_rank: int, producer_tp: int, consumer_tp: int, num_kv_heads: int) -> list[int]:
    """Consumer ranks that ``producer_rank`` sends to (ascending)."""
    return sorted({c.dst_rank for c in transfer_plan(producer_tp, consumer_tp, num_kv_heads)
                   if c.src_rank == producer_rank})


def source_ranks(consumer_rank: int, producer_tp: int, consumer_tp: int, num_kv_heads: int) -> list[int]:
    """Producer ranks that ``consumer_rank`` receives from (ascending)."""
    return sorted({c.src_rank for c in transfer_plan(producer_tp, consumer_tp, num_kv_heads)
                   if c.dst_rank == consumer_rank})


def validate_region_lengths(producer_lens: list[int], consumer_lens: list[int], producer_tp: int,
                            consumer_tp: int, num_kv_heads: int) -> str | None:
    """Check registered per-block K/V region lengths (bytes, one entry per
    region) against the TP split; returns an error message or None."""
    if len(producer_lens) != len(consumer_lens):
        return "producer and consumer register different numbers of KV regions"
    hp = head_shard(0, producer_tp, num_kv_heads).count
    hc = head_shard(0, consumer_tp, num_kv_heads).count
    for i, (lp, lc) in enumerate(zip(producer_lens, consumer_lens)):
        if lp % hp or lc % hc or lp // hp != lc // hc:
            return (f"KV region {i}: producer {lp} B over {hp} heads and consumer {lc} B over {hc} heads "
                    "do not have the same bytes per head")
    return None
