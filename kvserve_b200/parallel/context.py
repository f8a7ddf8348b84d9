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

Data-parallel replicas (``KVSERVE_REPLICAS=R`` or ``init_parallel(...,
replicas=R)``): the ``n`` ranks form ``R`` independent PD deployments of
``n/R`` ranks each (ranks ``[r*n/R, (r+1)*n/R)`` are replica ``r``), laid out
as above inside each replica.  The context's ``rank``, ``world_size``,
``peer_rank`` and groups are then replica-local, so the engine runs
unchanged; ``replica``, ``rank_offset`` (global rank of local rank 0) and
``job_cpu_group`` (all ranks) let a driver aggregate over replicas — the
role of the reference's per-``dp_rank`` Mooncake bootstrap
(kvsfuse-vllm0.30.0/mooncake/mooncake_connector.py:191-231).
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
    # data-parallel replicas (all defaults: one deployment over the whole job)
    replica: int = 0
    num_replicas: int = 1
    rank_offset: int = 0
    job_world_size: int = 0
    job_cpu_group: Optional[object] = None
    role_cpu_groups: Optional[dict] = None   # role -> gloo group of this replica's role ranks
    prefill_size: int = 0                     # prefill ranks per deployment (0: half; unequal = heterogeneous TP)

    @property
    def global_rank(self) -> int:
        return self.rank_offset + self.rank

    def global_ranks(self, role: str) -> list[int]:
        return [self.rank_offset + r for r in self.group_ranks(role)]

    @property
    def distributed(self) -> bool:
        return self.world_size > 1

    @property
    def is_prefill(self) -> bool:
        return self.role in ("prefill", "colocated")

    @property
    def is_decode(self) -> bool:
        return self.role in ("decode", "colocated")

    @property
    def num_prefill(self) -> int:
        """Ranks of the prefill group (the decode group has the others)."""
        return self.prefill_size or self.world_size // 2

    def group_ranks(self, role: str) -> list[int]:
        p = self.num_prefill
        return list(range(p)) if role == "prefill" else list(range(p, self.world_size))


def layout_for(rank: int, world_size: int, prefill: int = 0) -> tuple[str, int, int, int]:
    """(role, tp_rank, tp_size, peer_rank) of ``rank`` in a PD layout with
    ``prefill`` prefill ranks (0: half of them).  With unequal groups
    (heterogeneous TP) ``peer_rank`` is the rank of the other group with the
    same TP index modulo that group's size; the KV hand-off itself follows
    the head-range plan of :mod:`kvserve_b200.session.tp_plan`."""
    if world_size == 1:
        return "colocated", 0, 1, 0
    if not prefill:
        if world_size % 2:
            raise ValueError("a PD deployment of equal groups needs an even number of ranks")
        prefill = world_size // 2
    if not 1 <= prefill < world_size:
        raise ValueError(f"prefill ranks must be in [1, {world_size})")
    dec = world_size - prefill
    if rank < prefill:
        return "prefill", rank, prefill, prefill + rank % dec
    return "decode", rank - prefill, dec, (rank - prefill) % prefill


def init_parallel(backend: str = "nccl", timeout_s: float = 120.0, replicas: Optional[int] = None,
                  prefill: Optional[int] = None) -> ParallelContext:
    """Initialise torch.distributed from the torchrun environment (or a
    single-process context when WORLD_SIZE is unset / 1).  ``replicas``
    (default ``KVSERVE_REPLICAS`` or 1) splits the job into independent
    PD deployments; ``prefill`` (default ``KVSERVE_PREFILL_RANKS`` or half of
    a deployment) sizes its prefill group."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if replicas is None:
        replicas = int(os.environ.get("KVSERVE_REPLICAS", "1") or 1)
    if replicas < 1 or world % replicas:
        raise ValueError(f"{world} ranks do not split into {replicas} replicas")
    if prefill is None:
        prefill = int(os.environ.get("KVSERVE_PREFILL_RANKS", "0") or 0)
    if backend == "nccl" and torch.cuda.is_available():
        torch.cuda.set_device(local)
    if world == 1:
        return ParallelContext(job_world_size=1)
    if not dist.is_initialized():
        kwargs = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kwargs["device_id"] = torch.device("cuda", local)
        dist.init_process_group(**kwargs)
    td = datetime.timedelta(seconds=timeout_s)
    per = world // replicas
    mine = rank // per
    job_cpu = dist.new_group(list(range(world)), backend="gloo", timeout=td)
    ctx = None
    # every rank creates every group in the same order
    for r in range(replicas):
        off = r * per
        local_rank = rank - off
        if per == 1:
            if r == mine:
                ctx = ParallelContext(rank=0, world_size=1, local_rank=local, replica=r, num_replicas=replicas,
                                      rank_offset=off, job_world_size=world, job_cpu_group=job_cpu)
            continue
        npre = prefill or per // 2
        if not 1 <= npre < per or (not prefill and per % 2):
            raise ValueError(f"a deployment of {per} ranks can not have {npre} prefill ranks")
        groups, role_cpu = {}, {}
        for role in ("prefill", "decode"):
            ranks = [off + i for i in (range(npre) if role == "prefill" else range(npre, per))]
            groups[role] = dist.new_group(ranks, backend=backend) if len(ranks) > 1 else None
            role_cpu[role] = dist.new_group(ranks, backend="gloo", timeout=td)
        rep_ranks = list(range(off, off + per))
        cpu = job_cpu if replicas == 1 else dist.new_group(rep_ranks, backend="gloo", timeout=td)
        wg = dist.group.WORLD if replicas == 1 else dist.new_group(rep_ranks, backend=backend)
        if r == mine:
            role, tp_rank, tp_size, peer = layout_for(local_rank, per, npre)
            ctx = ParallelContext(rank=local_rank, world_size=per, local_rank=local, role=role, tp_rank=tp_rank,
                                  tp_size=tp_size, peer_rank=peer, tp_group=groups[role], cpu_group=cpu,
                                  world_group=wg, replica=r, num_replicas=replicas, rank_offset=off,
                                  job_world_size=world, job_cpu_group=job_cpu, role_cpu_groups=role_cpu,
                                  prefill_size=npre)
    return ctx


def destroy_parallel(ctx: ParallelContext) -> None:
    if (ctx.distributed or ctx.job_world_size > 1) and dist.is_initialized():
        dist.destroy_process_group()
