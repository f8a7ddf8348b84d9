"""Fixed-profile KV compression runtime, API version 1 (the surface of
kvserve_v1/compression/runtime/__init__.py): transport-independent, the
caller owns cache registration, slot scheduling and the network."""
from __future__ import annotations

import os

from .config import CompressionConfig
from .memory import CompressionMemoryPlan, build_memory_plan
from .spec import CacheSpec

API_VERSION = 1


def create_runtime(plan: CompressionMemoryPlan, kv_cache_layout: str = "HND", blocks_per_logical: int = 1,
                   device=None, backend: str = "auto", **kwargs):
    """Create the runtime for ``plan``.  ``backend`` is accepted for API
    compatibility: every backend name runs the sm_100a fused frame kernels
    (there is one implementation, no dispatch)."""
    if backend == "auto":
        # the reference's selector variable (auto / python / cpp) is accepted;
        # every choice runs the same kernels
        env = os.environ.get("KVSERVE_COMPRESSION_BACKEND", "auto").strip().lower()
        if env not in ("auto", "python", "cpp", "fused", "standard"):
            raise ValueError(f"KVSERVE_COMPRESSION_BACKEND must be auto, python or cpp, got {env!r}")
    if backend not in ("auto", "fused", "standard"):
        raise ValueError("backend must be auto, fused or standard")
    from .manager import CompressionRuntime
    kwargs.pop("standard_backend", None)
    return CompressionRuntime(plan, kv_cache_layout, blocks_per_logical, device, **kwargs)


def __getattr__(name):
    if name in ("CompressionRuntime", "EncodeResult"):
        from . import manager
        return getattr(manager, name)
    raise AttributeError(name)


__all__ = ["API_VERSION", "CacheSpec", "CompressionConfig", "CompressionRuntime", "build_memory_plan",
           "create_runtime", "CompressionMemoryPlan"]
