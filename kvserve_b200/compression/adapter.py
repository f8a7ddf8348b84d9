"""Connector-facing compression adapter (behaviour of
kvserve_v1/compression/manager.py:54-345).

Three modes, selected by ``kv_connector_extra_config["compression"]``:
``"default"`` (built-in profile, model name patched to the running model),
a custom pipeline dict, or ``{"mode": "controller", "library_path": ...,
"service_config": {...}}`` (online profile selection; the chosen profile is
embedded in the payload metadata as ``ctrl_profile_cfg`` so the receiver can
rebuild the same pipeline).

Fused normalisation: a pipeline whose quantizer is the fused Hadamard
operator (``impl: "tilelang_fused"``) drops its separate Hadamard stage and
keeps its seed; a non-Hadamard transform or conflicting seeds are rejected.
"""
from __future__ import annotations

import json
import logging
import time
from typing import Any, Optional

import torch

from .manager import (CompressedKVData, CompressionConfig, CompressionManager, get_default_compression_config)

log = logging.getLogger("kvserve_b200.adapter")

COMPRESSED_SENTINEL = "__compressed__"


def is_compressed_layer_names(names: list[str]) -> bool:
    return bool(names) and names[0] == COMPRESSED_SENTINEL


def strip_sentinel(names: list[str]) -> list[str]:
    return names[1:] if is_compressed_layer_names(names) else names


def add_sentinel(names: list[str]) -> list[str]:
    return [COMPRESSED_SENTINEL] + list(names)


def _key(cfg: dict) -> str:
    return json.dumps(cfg, sort_keys=True, default=str)


class KVCompressionAdapter:
    CONTEXT_TTL_S = 300.0

    def __init__(self, compression_spec: Any, num_kv_heads: int, head_size: int, model_name: Optional[str] = None,
                 tp_rank: int = 0, tp_size: int = 1, num_layers: int = 0):
        self._num_kv_heads, self._head_size = num_kv_heads, head_size
        self._model_name, self._tp_rank, self._tp_size = model_name, tp_rank, tp_size
        self._num_layers = num_layers
        self._controller = None
        self._service_cfg: dict = {}
        self._last_contexts: dict[str, tuple[float, dict]] = {}
        self._cache: dict[str, tuple[CompressionManager, CompressionConfig]] = {}
        if compression_spec == "default":
            cfg = get_default_compression_config()
            if model_name and "quantizer_config" in cfg:
                cfg["quantizer_config"]["model_name"] = model_name
            self._manager, self._config = self._build(cfg), self._make_config(cfg)
        elif isinstance(compression_spec, dict) and compression_spec.get("mode") == "controller":
            self._init_controller(compression_spec)
            self._manager, self._config = None, None
        else:
            self._manager, self._config = self._build(compression_spec), self._make_config(compression_spec)

    # ------------------------------------------------------------- config
    def _init_controller(self, spec: dict) -> None:
        from .controller import OnlineController, ProfileLibrary
        self._controller = OnlineController(ProfileLibrary(spec["library_path"]), epsilon=spec.get("epsilon", 0.1),
                                            alpha=spec.get("alpha", 0.2))
        self._service_cfg = spec.get("service_config", {})

    @staticmethod
    def is_fused(cfg: dict) -> bool:
        if cfg.get("impl") == "tilelang_fused" or cfg.get("quantizer_impl") == "tilelang_fused":
            return True
        return (cfg.get("quantizer_config") or {}).get("impl") == "tilelang_fused"

    @classmethod
    def normalize_config(cls, cfg: dict) -> dict:
        cfg = dict(cfg)
        if not cls.is_fused(cfg):
            return cfg
        if (cfg.get("quantizer_config") or {}).get("impl") == "centered_codebook":
            raise ValueError("centered_codebook cannot use the fused implementation")
        pipeline = list(cfg.get("pipeline", []))
        if "quantizer" not in pipeline:
            raise ValueError("the fused quantizer requires a quantizer pipeline stage")
        qc = dict(cfg.get("quantizer_config") or {})
        qc["impl"] = "tilelang_fused"
        if "transformer" in pipeline:
            tc = dict(cfg.get("transformer_config") or {})
            if tc.get("transform_type", "hadamard") != "hadamard":
                raise ValueError("the fused quantizer only fuses the Hadamard transformer")
            seed = tc.get("seed", 0x3333)
            explicit = qc.get("base_seed", qc.get("seed"))
            if "seed" in tc and explicit is not None and int(explicit) != int(seed):
                raise ValueError("Conflicting transformer seed and fused quantizer seed")
            qc.setdefault("base_seed", explicit if explicit is not None else seed)
            pipeline = [p for p in pipeline if p != "transformer"]
        cfg["quantizer_config"] = qc
        cfg["pipeline"] = pipeline
        return cfg

    def _make_config(self, cfg: dict) -> CompressionConfig:
        cfg = self.normalize_config(cfg)
        qc = cfg.get("quantizer_config")
        if qc is not None:
            qc = dict(qc)
            qc["tp_rank"] = self._tp_rank
            qc["tensor_parallel_size"] = self._tp_size
        return CompressionConfig(enabled=cfg.get("enabled", True), pipeline=cfg.get("pipeline", []),
                                 transformer_config=cfg.get("transformer_config"), quantizer_config=qc,
                                 codec_config=cfg.get("codec_config"), min_compress_size=cfg.get("min_compress_size", 0))

    def _build(self, cfg: dict) -> CompressionManager:
        cfg = self.normalize_config(cfg)
        pipeline = list(cfg.get("pipeline", []))
        t_cls = q_cls = c_cls = None
        if "transformer" in pipeline:
            from .transformer import KVServeTransformer
            t_cls = KVServeTransformer
        if "quantizer" in pipeline:
            impl = (cfg.get("quantizer_config") or {}).get("impl")
            if self.is_fused(cfg):
                from .quantizer import FusedHadamardQuantizer as q_cls
            elif impl == "centered_codebook":
                from .quantizer import CenteredCodebookQuantizer as q_cls
            else:
                from .quantizer import KVServeQuantizer as q_cls
        if "codec" in pipeline:
            from .codec import KVServeCodec as c_cls
        config = self._make_config(cfg)
        if config.quantizer_config is not None and self._num_layers:
            config.quantizer_config.setdefault("num_layers", self._num_layers)
            config.quantizer_config.setdefault("num_kv_heads", self._num_kv_heads * self._tp_size)
        return CompressionManager(config, t_cls, q_cls, c_cls)

    def _cached(self, cfg: dict) -> tuple[CompressionManager, CompressionConfig]:
        k = _key(cfg)
        if k not in self._cache:
            self._cache[k] = (self._build(cfg), self._make_config(cfg))
        return self._cache[k]

    # ---------------------------------------------------------------- API
    def compress(self, stacked_kv: torch.Tensor, request_id: str) -> Optional[CompressedKVData]:
        meta = {"original_dtype": str(stacked_kv.dtype).replace("torch.", ""),
                "original_shape": list(stacked_kv.shape)}
        if stacked_kv.ndim == 6:
            x6 = stacked_kv.contiguous()
        elif stacked_kv.ndim == 4:
            L, _, T, _ = stacked_kv.shape
            x6 = stacked_kv.contiguous().view(L, 2, 1, T, self._num_kv_heads, self._head_size)
        else:
            raise ValueError(f"Unsupported KV tensor rank for compression: {stacked_kv.ndim}")
        if self._controller is not None:
            return self._compress_controller(x6, request_id, meta)
        return self._manager.compress_all_layers(x6, request_id, self._config, meta)

    def decompress(self, compressed: CompressedKVData) -> Optional[torch.Tensor]:
        if self._controller is not None:
            cfg = compressed.metadata.get("ctrl_profile_cfg")
            if cfg is None:
                log.error("controller mode: ctrl_profile_cfg missing from metadata")
                return None
            manager, config = self._cached(cfg)
        else:
            manager, config = self._manager, self._config
        res = manager.decompress_all_layers(compressed, config)
        if res is None:
            return None
        if isinstance(res, list):
            res = torch.cat(res, dim=0)
        shape = compressed.metadata.get("original_shape")
        if shape is not None:
            return res.contiguous().view(*[int(x) for x in shape])
        return res.contiguous().view(res.shape[0], 2, -1, self._num_kv_heads * self._head_size)

    def update_controller(self, request_id: str, observed_latency_ms: float) -> None:
        if self._controller is None:
            return
        entry = self._last_contexts.pop(request_id, None)
        if entry is not None:
            self._controller.update(entry[1], observed_latency_ms)

    def get_controller_stats(self) -> Optional[dict]:
        return None if self._controller is None else self._controller.get_statistics()

    def _evict(self) -> None:
        cutoff = time.monotonic() - self.CONTEXT_TTL_S
        for rid in [r for r, (ts, _) in self._last_contexts.items() if ts < cutoff]:
            self._last_contexts.pop(rid)

    def _compress_controller(self, x6: torch.Tensor, request_id: str, meta: dict) -> Optional[CompressedKVData]:
        V = float(x6.numel() * x6.element_size())
        sc = self._service_cfg
        profile, context = self._controller.select_profile(
            V, float(sc.get("bandwidth_mbps", 10_000.0)), float(sc.get("t_model_ms", 0.0)),
            float(sc.get("slo_ms", float("inf"))), float(sc.get("accuracy_requirement", 0.9)))
        self._last_contexts[request_id] = (time.monotonic(), context)
        self._evict()
        if profile is None:
            return None
        meta["ctrl_profile_cfg"] = profile.compression_config
        manager, config = self._cached(profile.compression_config)
        return manager.compress_all_layers(x6, request_id, config, meta)
