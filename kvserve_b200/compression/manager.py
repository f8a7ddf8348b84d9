"""Modular compression pipeline (behaviour of
kvserve_v1/compression/compression_manager.py).

``compress_all_layers`` runs, per layer, transform -> quantize into a stacked
codec buffer and then ONE codec call over the whole buffer:

* codec byte order ``"permuted"`` ``[L, 2, H, B, S, D]`` (default) or
  ``"native"`` ``[L, 2, B, S, H, D]`` (``KVSERVE_CODEC_LAYOUT``);
* quantizers that accept ``out=`` write symbols straight into the buffer
  (no transform stage in that case);
* payloads above 500 MiB are compressed in 8-layer chunks;
* a codec failure falls back to the raw bytes and is recorded
  (``codec_skipped`` / ``codec_error``);
* payloads below ``min_compress_size`` are not compressed (``None``).

``decompress_all_layers`` mirrors it (chunked payloads return a list).
"""
from __future__ import annotations

import copy
import logging
import os
from dataclasses import dataclass, field
from typing import Any, Optional

import torch

from .components import Codec, Quantizer, Transformer

log = logging.getLogger("kvserve_b200.compression")

_LAYOUT_ENV = "KVSERVE_CODEC_LAYOUT"
CHUNK_THRESHOLD_BYTES = 500 * 1024 * 1024
CHUNK_LAYERS = 8

DEFAULT_COMPRESSION_CONFIG: dict[str, Any] = {
    "enabled": True,
    "pipeline": ["quantizer", "codec"],
    "quantizer_config": {
        "model_name": "Llama-3.1-8B-Instruct",
        "hybrid_ratio": 0.8,
        "high_key_max_value": 12,
        "high_value_max_value": 8,
        "low_key_max_value": 6,
        "low_value_max_value": 4,
        "axis_key": "channel",
        "axis_value": "token",
        "split_type": "head",
    },
    "codec_config": {"codec_type": "nvcomp", "nvcomp_algorithm": "ANS", "data_type": "|u1"},
    "min_compress_size": 1024,
}


def get_default_compression_config() -> dict[str, Any]:
    return copy.deepcopy(DEFAULT_COMPRESSION_CONFIG)


@dataclass
class CompressionConfig:
    enabled: bool = False
    transformer_config: Optional[dict] = None
    quantizer_config: Optional[dict] = None
    codec_config: Optional[dict] = None
    pipeline: Optional[list] = None
    min_compress_size: int = 0


@dataclass
class CompressedKVData:
    request_id: str
    layer_id: int
    compressed_tensor: Optional[torch.Tensor] = None
    metadata: Optional[dict] = None
    original_size: int = 0
    compressed_size: int = 0
    is_chunked: bool = False
    chunks: Optional[list] = None
    chunk_metadata: Optional[list] = None


def codec_layout() -> str:
    v = os.environ.get(_LAYOUT_ENV, "permuted").strip().lower()
    return v if v in ("native", "permuted") else "permuted"


def _dtype_name(dtype: torch.dtype) -> str:
    return str(dtype).replace("torch.", "")


class CompressionManager:
    def __init__(self, config: CompressionConfig, transformer=None, quantizer=None, codec=None):
        self.config = config
        self.transformer: Optional[Transformer] = transformer(**(config.transformer_config or {})) if transformer else None
        self.quantizer: Optional[Quantizer] = quantizer(**(config.quantizer_config or {})) if quantizer else None
        self.codec: Optional[Codec] = codec(**(config.codec_config or {})) if codec else None
        self.original_size = 0
        self.compressed_size = 0
        if config.enabled and config.pipeline:
            for name in config.pipeline:
                if getattr(self, name, None) is None:
                    raise ValueError(f"{name} component required but not provided")

    def update_config(self, config: CompressionConfig) -> None:
        self.config = config
        if self.transformer is not None:
            self.transformer.update_params(**(config.transformer_config or {}))
        if self.quantizer is not None:
            self.quantizer.update_params(**(config.quantizer_config or {}))
        if self.codec is not None:
            self.codec.update_params(**(config.codec_config or {}))

    # ------------------------------------------------------------- helpers
    def _uses(self, stage: str) -> bool:
        return stage in (self.config.pipeline or [])

    def _direct(self) -> bool:
        return (self._uses("quantizer") and not self._uses("transformer")
                and bool(getattr(self.quantizer, "supports_out_buffer", False)))

    def _process_layers(self, data: torch.Tensor, start: int, qparams: list, meta: dict,
                        layout: str) -> torch.Tensor:
        L = data.shape[0]
        if self._direct():
            meta["quantization_applied"] = True
            native = torch.empty(data.shape, dtype=torch.uint8, device=data.device)
            for i in range(L):
                _, qp = self.quantizer.quantize(start + i, data[i], out=native[i], **(self.config.quantizer_config or {}))
                qparams.append(qp)
            return native if layout == "native" else native.permute(0, 1, 4, 2, 3, 5).contiguous()
        buf = None
        for i in range(L):
            x = data[i]
            if self._uses("transformer"):
                x = self.transformer.transform(start + i, x, **(self.config.transformer_config or {}))
                meta["transformer_applied"] = True
            if self._uses("quantizer"):
                x, qp = self.quantizer.quantize(start + i, x, **(self.config.quantizer_config or {}))
                qparams.append(qp)
                meta["quantization_applied"] = True
            if buf is None:
                shape = (x.shape[0], x.shape[3], x.shape[1], x.shape[2], x.shape[4]) if layout == "permuted" \
                    else tuple(x.shape)
                buf = torch.empty((L,) + shape, dtype=x.dtype, device=x.device)
            buf[i].copy_(x.permute(0, 3, 1, 2, 4) if layout == "permuted" else x)
        return buf

    def _encode(self, buf: torch.Tensor, meta: dict, layer_id: int, request_id: str) -> torch.Tensor:
        if self._uses("codec"):
            try:
                out = self.codec.encode(layer_id, buf, **(self.config.codec_config or {}))
                meta["codec_applied"] = True
                return out
            except Exception as exc:  # codec failure -> raw bytes
                log.warning("codec failed for %s: %s: %s", request_id, type(exc).__name__, exc)
                meta["codec_skipped"] = True
                meta["codec_error"] = f"{type(exc).__name__}: {exc}"
        return buf.reshape(-1).view(torch.uint8).contiguous()

    def _decode(self, payload: torch.Tensor, meta: dict, layer_id: int) -> torch.Tensor:
        dtype, shape = meta["codec_dtype"], meta["codec_shape"]
        if self._uses("codec") and meta.get("codec_applied", False):
            return self.codec.decode(layer_id, payload, dtype, shape, meta.get("device", str(payload.device)),
                                     **(self.config.codec_config or {}))
        return payload.view(getattr(torch, dtype)).reshape(shape)

    # ----------------------------------------------------------- compress
    def compress_all_layers(self, all_layers_data: torch.Tensor, request_id: str, config: CompressionConfig,
                            metadata: dict) -> Optional[CompressedKVData]:
        self.update_config(config)
        if not self.config.enabled or not self.config.pipeline:
            return None
        if not isinstance(all_layers_data, torch.Tensor) or all_layers_data.dim() != 6:
            log.error("all_layers_data must be a 6-D tensor [L, 2, B, S, H, D]")
            return None
        try:
            L = all_layers_data.shape[0]
            original = all_layers_data.numel() * all_layers_data.element_size()
            if original < self.config.min_compress_size:
                return None
            if original > CHUNK_THRESHOLD_BYTES:
                return self._compress_chunked(all_layers_data, request_id, metadata)
            meta = {"request_id": request_id, "original_dtype": _dtype_name(all_layers_data.dtype),
                    "original_size": original, "device": str(all_layers_data.device), "start_layer_id": 0,
                    "num_layers": L, **metadata}
            layout = codec_layout()
            meta["codec_layout"] = layout
            qparams: list = []
            buf = self._process_layers(all_layers_data, 0, qparams, meta, layout)
            if self._uses("quantizer"):
                meta["quantization_params"] = qparams
            meta["codec_shape"] = list(buf.shape)
            meta["codec_dtype"] = _dtype_name(buf.dtype)
            payload = self._encode(buf, meta, L - 1, request_id)
            self.original_size = original
            self.compressed_size = payload.numel() * payload.element_size()
            meta["compressed_size"] = self.compressed_size
            return CompressedKVData(request_id, L - 1, payload, meta, original, self.compressed_size)
        except Exception:
            log.exception("compression failed for %s", request_id)
            return None

    def _compress_chunked(self, data: torch.Tensor, request_id: str, metadata: dict) -> CompressedKVData:
        L = data.shape[0]
        chunks, metas = [], []
        layout = codec_layout()
        total = 0
        for start in range(0, L, CHUNK_LAYERS):
            part = data[start:start + CHUNK_LAYERS]
            meta = {"request_id": request_id, "original_dtype": _dtype_name(data.dtype),
                    "device": str(data.device), "start_layer_id": start, "num_layers": part.shape[0],
                    "codec_layout": layout, **metadata}
            qparams: list = []
            buf = self._process_layers(part, start, qparams, meta, layout)
            if self._uses("quantizer"):
                meta["quantization_params"] = qparams
            meta["codec_shape"] = list(buf.shape)
            meta["codec_dtype"] = _dtype_name(buf.dtype)
            payload = self._encode(buf, meta, start + part.shape[0] - 1, request_id)
            total += payload.numel() * payload.element_size()
            chunks.append(payload)
            metas.append(meta)
        original = data.numel() * data.element_size()
        head = {"request_id": request_id, "original_dtype": _dtype_name(data.dtype), "original_size": original,
                "num_layers": L, "chunk_layers": CHUNK_LAYERS, **metadata}
        self.original_size, self.compressed_size = original, total
        return CompressedKVData(request_id, L - 1, None, head, original, total, True, chunks, metas)

    # --------------------------------------------------------- decompress
    def _restore_layers(self, payload: torch.Tensor, meta: dict) -> torch.Tensor:
        L = int(meta["num_layers"])
        start = int(meta.get("start_layer_id", 0))
        cur = self._decode(payload, meta, start + L - 1)
        if meta.get("codec_layout", "permuted") == "permuted":
            cur = cur.permute(0, 1, 3, 4, 2, 5).contiguous()
        dtype = getattr(torch, meta.get("original_dtype", "bfloat16"))
        out = torch.empty(cur.shape, dtype=dtype, device=cur.device)
        qps = meta.get("quantization_params")
        for i in range(L):
            x = cur[i]
            if self._uses("quantizer"):
                x = self.quantizer.dequantize(start + i, x, qps[i], **(self.config.quantizer_config or {}))
            if self._uses("transformer"):
                x = self.transformer.inverse(start + i, x, **(self.config.transformer_config or {}))
            out[i].copy_(x.to(dtype))
        return out

    def decompress_all_layers(self, compressed: CompressedKVData, config: CompressionConfig):
        self.update_config(config)
        if not self.config.enabled or not self.config.pipeline:
            return None
        try:
            if compressed.is_chunked:
                return [self._restore_layers(c, m) for c, m in zip(compressed.chunks, compressed.chunk_metadata)]
            return self._restore_layers(compressed.compressed_tensor, compressed.metadata)
        except Exception:
            log.exception("decompression failed for %s", compressed.request_id)
            return None
