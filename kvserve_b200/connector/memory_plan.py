"""Connector-owned GPU memory planned before KV-cache sizing (the interface
the reference adds to vLLM: kvsfuse-vllm0.30.0 ``base.py:86-104,219-226,306-310``
and ``gpu_worker.py:703-724,797-801``).

A worker asks the connector class for a :class:`KVConnectorWorkerMemoryPlan`
*before* it sizes the KV cache (``reserved_bytes`` is taken off the memory
budget), then hands the same plan to the connector instance *after* the KV
cache exists (``initialize_worker_memory``), which allocates exactly what was
planned.  Stock vLLM does not call these hooks; :func:`adjusted_utilization`
converts a plan into the ``gpu_memory_utilization`` to pass instead, so the
reservation also works unpatched.

The plan's ``connector_data`` is this framework's
:class:`~kvserve_b200.compression.runtime.CompressionMemoryPlan` (frame
arena per receive slot, lossless-codec capacity and scratch), built from the
same fixed profile the runtime later runs.
"""
from __future__ import annotations

import re
from dataclasses import dataclass, field
from typing import Any, Mapping, Optional

import torch

from ..compression.runtime import CacheSpec, CompressionConfig, build_memory_plan


@dataclass(frozen=True)
class KVConnectorWorkerMemoryPlan:
    """GPU memory a worker-side connector reserves before KV sizing."""

    reserved_bytes: int = 0
    connector_data: Any = None


@dataclass
class KVConnectorTransferResults:
    """Asynchronous transfer completions of one worker snapshot; failed
    receives are also listed in ``finished_recving`` so the scheduler can
    release the request from its wait state."""

    finished_sending: set = field(default_factory=set)
    finished_recving: set = field(default_factory=set)
    failed_recving: set = field(default_factory=set)


_LAYER_RE = re.compile(r"(\d+)(?!.*\d)")


def layer_index_of(name: str) -> int:
    """Layer index of a vLLM attention layer name (its last integer)."""
    m = _LAYER_RE.search(name)
    if m is None:
        raise ValueError(f"no layer index in {name!r}")
    return int(m.group(1))


def cache_specs_from_vllm(kv_cache_specs: Mapping[str, Any]) -> dict[str, CacheSpec]:
    """Map vLLM ``KVCacheSpec`` objects (anything with ``block_size``,
    ``num_kv_heads``, ``head_size`` and ``dtype``) to runtime cache specs."""
    out = {}
    for name, s in kv_cache_specs.items():
        hv = getattr(s, "head_size_v", None)
        out[name] = CacheSpec(layer_index_of(name), int(s.block_size), int(s.num_kv_heads), int(s.head_size),
                              getattr(s, "dtype", torch.bfloat16), int(hv) if hv else None)
    return out


def plan_worker_memory(extra_config: Optional[Mapping[str, Any]], kv_cache_specs: Mapping[str, Any],
                       tp_rank: int = 0, tp_size: int = 1) -> KVConnectorWorkerMemoryPlan:
    """The plan for ``kv_connector_extra_config``: nothing when the runtime
    is disabled, else the runtime's slot arenas plus metadata and guard."""
    cfg = CompressionConfig.from_extra_config(dict(extra_config or {}))
    if not cfg.enabled or not kv_cache_specs:
        return KVConnectorWorkerMemoryPlan()
    plan = build_memory_plan(cfg, cache_specs_from_vllm(kv_cache_specs), tp_size=tp_size, tp_rank=tp_rank)
    return KVConnectorWorkerMemoryPlan(int(plan.reserved_bytes), plan)


def adjusted_utilization(total_bytes: int, gpu_memory_utilization: float,
                         plan: KVConnectorWorkerMemoryPlan) -> float:
    """``gpu_memory_utilization`` that leaves ``plan.reserved_bytes`` free
    on a device of ``total_bytes`` (for engines that do not call the plan
    hooks)."""
    if total_bytes <= 0:
        raise ValueError("total_bytes must be positive")
    budget = gpu_memory_utilization * total_bytes - plan.reserved_bytes
    if budget <= 0:
        raise ValueError("the connector reservation exceeds the memory budget")
    return budget / total_bytes


class WorkerMemory:
    """Allocation made by ``initialize_worker_memory``: one device buffer of
    exactly the planned size (carved by the runtime), or nothing."""

    def __init__(self, plan: Optional[KVConnectorWorkerMemoryPlan], device=None):
        self.plan = plan or KVConnectorWorkerMemoryPlan()
        self.buffer: Optional[torch.Tensor] = None
        if self.plan.reserved_bytes > 0:
            dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
            self.buffer = torch.empty(self.plan.reserved_bytes, dtype=torch.uint8, device=dev)

    @property
    def nbytes(self) -> int:
        return 0 if self.buffer is None else self.buffer.numel()
