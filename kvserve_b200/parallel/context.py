"""Process layout of a disaggregated prefill/decode deployment on one node.

One process per GPU.  With ``n`` ranks:

* ``n == 1``: *colocated* — the single rank runs prefill and decode on one GPU
  (the KV hand-off is a device-local frame write + decode).
* ``n >= 2`` (even): ranks ``[0, n/2)`` form the prefill group (tensor
  parallel of size n/2) and ranks ``[n/2, n)`` the decode group.  Prefill
  rank ``i`` hands its KV shard to decode rank ``n/2 + i`` (one channel per
  TP rank, as kvserve_v1/transport/nccl_transport.py:96 opens one channel
  per ``kv_port + tp_rank``).

Collectives inside a group use NCCL (NVLink / NVSwitch); small host objects
(IPC handles, control messages) go over a gloo group.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class ParallelContext:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    role: str = "colocated"          # colocated | prefill | decode
    tp_rank: int = 0
    tp_size: int = 1
    peer_rank: int = 0               # paired rank in the other role
    tp_group: Optional[object] = None
    cpu_group: Optional[object] = None
    world_group: Optional[object] = None

    @property
    def distributed(self) -> bool:
        return self.world_size > 1

    @property
    def is_prefill(self) -> bool:
        return self.role in ("prefill", "colocated")

    @property
    def is_decode(self) -> bool:
        return self.role in ("decode", "colocated")

    def group_ranks(self, role: str) -> list[int]:
        half = self.world_size // 2
        return list(range(half)) if role == "prefill" else list(range(half, self.world_size))


def layout_for(rank: int, world_size: int) -> tuple[str, int, int, int]:
    """(role, tp_rank, tp_size, peer_rank) of ``rank`` in a PD layout."""
    if world_size == 1:
        return "colocated", 0, 1, 0
    if world_size % 2:
        raise ValueError("a PD deployment needs an even number of ranks (P and D groups of equal TP)")
    half = world_size // 2
    if rank < half:
        return "prefill", rank, half, rank + half
    return "decode", rank - half, half, rank - half


def init_parallel(backend: str = "nccl", timeout_s: float = 120.0) -> ParallelContext:
    """Initialise torch.distributed from the torchrun environment (or a
    single-process context when WORLD_SIZE is unset / 1)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if backend == "nccl" and torch.cuda.is_available():
        torch.cuda.set_device(local)
    if world == 1:
        return ParallelContext()
    if not dist.is_initialized():
        kwargs = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(**kwargs)
    role, tp_rank, tp_size, peer = layout_for(rank, world)
    half = world // 2
    groups = {}
    # every rank must create every group in the same order
    for r in ("prefill", "decode"):
        ranks = list(range(half)) if r == "prefill" else list(range(half, world))
        groups[r] = dist.new_group(ranks, backend=backend) if tp_size > 1 else None
    cpu = dist.new_group(list(range(world)), backend="gloo", timeout=datetime.timedelta(seconds=timeout_s))
    return ParallelContext(rank=rank, world_size=world, local_rank=local, role=role, tp_rank=tp_rank,
                           tp_size=tp_size, peer_rank=peer, tp_group=groups[role], cpu_group=cpu,
                           world_group=dist.group.WORLD)


def destroy_parallel(ctx: ParallelContext) -> None:
    if ctx.distributed and dist.is_initialized():
        dist.destroy_process_group()
