"""Fixed-profile KV compression runtime, API version 1 (the surface of
kvserve_v1/compression/runtime/__init__.py): transport-independent, the
caller owns cache registration, slot scheduling and the network."""
from __future__ import annotations

import os

import torch

from .config import CompressionConfig
from .memory import CompressionMemoryPlan, build_memory_plan
from .spec import CacheSpec

API_VERSION = 1


def create_runtime(plan: CompressionMemoryPlan, kv_cache_layout: str = "HND", blocks_per_logical: int = 1,
                   device=None, backend: str = "auto", **kwargs):
    """Create the runtime for ``plan``.  ``backend`` is accepted for API
    compatibility: every backend name runs the sm_100a fused frame kernels
    on a GPU; a CPU ``device`` gets the same API on the frame format's CPU
    reference encoder and decoder (:mod:`.cpu_runtime`)."""
    if backend == "auto":
        # the reference's selector variable (auto / python / cpp) is accepted;
        # every choice runs the same kernels
        env = os.environ.get("KVSERVE_COMPRESSION_BACKEND", "auto").strip().lower()
        if env not in ("auto", "python", "cpp", "fused", "standard"):
            raise ValueError(f"KVSERVE_COMPRESSION_BACKEND must be auto, python or cpp, got {env!r}")
    if backend not in ("auto", "fused", "standard"):
        raise ValueError("backend must be auto, fused or standard")
    kwargs.pop("standard_backend", None)
    if device is not None and torch.device(device).type == "cpu":
        from .cpu_runtime import CpuCompressionRuntime
        return CpuCompressionRuntime(plan, kv_cache_layout, blocks_per_logical, device, **kwargs)
    from .manager import CompressionRuntime
    return CompressionRuntime(plan, kv_cache_layout, blocks_per_logical, device, **kwargs)


def __getattr__(name):
    if name in ("CompressionRuntime", "EncodeResult"):
        from . import manager
        return getattr(manager, name)
    raise AttributeError(name)


__all__ = ["API_VERSION", "CacheSpec", "CompressionConfig", "CompressionRuntime", "build_memory_plan",
           "create_runtime", "CompressionMemoryPlan"]
