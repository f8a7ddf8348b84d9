"""Fixed-profile runtime configuration (public keys and validation of
kvserve_v1/compression/runtime/config.py:17-221).

``CompressionConfig.from_extra_config(extra)`` reads
``extra["compression"]`` (public switch ``"enable-compression-pipeline"``)
or the lossless aggregate transport ``extra["raw_aggregate"]`` /
``extra["raw_agg"]`` (``true`` or ``{slot_count, logical_blocks_per_chunk}``),
which takes precedence over compression settings.
"""
from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Any, Literal

log = logging.getLogger("kvserve_b200.runtime")

RAW_AGGREGATE_KEY = "raw_aggregate"
RAW_AGGREGATE_ALIAS = "raw_agg"
RAW_AGGREGATE_SLOT_COUNT = 2
RAW_AGGREGATE_LOGICAL_BLOCKS_PER_CHUNK = 160
_WARNED = [False]


def _parse_raw_aggregate(extra: dict) -> tuple[int, int] | None:
    if RAW_AGGREGATE_KEY in extra:
        raw = extra[RAW_AGGREGATE_KEY]
    elif RAW_AGGREGATE_ALIAS in extra:
        raw = extra[RAW_AGGREGATE_ALIAS]
    else:
        return None
    if raw is None or raw is False:
        return None
    if raw is True:
        raw = {}
    if not isinstance(raw, dict):
        raise ValueError(f"{RAW_AGGREGATE_KEY} must be true or an object with slot_count/logical_blocks_per_chunk")
    unknown = set(raw) - {"slot_count", "logical_blocks_per_chunk"}
    if unknown:
        raise ValueError(f"Unknown {RAW_AGGREGATE_KEY} parameters: {sorted(unknown)}")
    slots = int(raw.get("slot_count", RAW_AGGREGATE_SLOT_COUNT))
    lbpc = int(raw.get("logical_blocks_per_chunk", RAW_AGGREGATE_LOGICAL_BLOCKS_PER_CHUNK))
    if slots < 1:
        raise ValueError(f"{RAW_AGGREGATE_KEY}.slot_count must be >= 1")
    if lbpc < 1:
        raise ValueError(f"{RAW_AGGREGATE_KEY}.logical_blocks_per_chunk must be >= 1")
    return slots, lbpc


@dataclass(frozen=True)
class CompressionConfig:
    enabled: bool = False
    transport: Literal["raw", "compression", "raw_aggregate"] = "compression"
    transformer: Literal["hadamard"] = "hadamard"
    seed: int = 3237919422
    split_type: Literal["head", "layer"] = "layer"
    score_path: str | None = None
    hybrid_ratio: float = 0.8
    axis_key: Literal["channel", "token", "tensor"] = "channel"
    axis_value: Literal["channel", "token", "tensor"] = "token"
    high_key_num_levels: int = 12
    high_value_num_levels: int = 8
    low_key_num_levels: int = 6
    low_value_num_levels: int = 4
    codec: Literal["ans"] = "ans"
    slot_count: int = 2
    logical_blocks_per_chunk: int = 1
    pipeline: tuple = ("transformer", "quantizer", "codec")

    @property
    def available(self) -> bool:
        return self.enabled

    @property
    def is_raw_aggregate(self) -> bool:
        return self.transport == "raw_aggregate"

    @property
    def uses_aggregate(self) -> bool:
        return "aggregate" in self.pipeline

    @property
    def uses_transformer(self) -> bool:
        return not self.uses_aggregate and "transformer" in self.pipeline

    @property
    def uses_quantizer(self) -> bool:
        return not self.uses_aggregate and "quantizer" in self.pipeline

    @property
    def uses_codec(self) -> bool:
        return not self.uses_aggregate and "codec" in self.pipeline

    @classmethod
    def from_extra_config(cls, extra_config: dict[str, Any]) -> "CompressionConfig":
        extra = extra_config or {}
        agg = _parse_raw_aggregate(extra)
        if agg is not None:
            comp = extra.get("compression") or {}
            if comp.get("enable-compression-pipeline", False) and not _WARNED[0]:
                _WARNED[0] = True
                log.warning("raw_aggregate transport selected; ignoring compression parameters: %s",
                            ", ".join(sorted(str(k) for k in comp)))
            return cls(enabled=True, transport="raw_aggregate", pipeline=("aggregate",), slot_count=agg[0],
                       logical_blocks_per_chunk=agg[1])
        raw = extra.get("compression") or {}
        if not raw.get("enable-compression-pipeline", False):
            return cls(enabled=False, transport="raw")
        norm = dict(raw)
        norm.pop("enable-compression-pipeline")
        if "pipeline" in norm:
            norm["pipeline"] = tuple(norm["pipeline"])
        cfg = cls(enabled=True, transport="compression", **norm)
        cfg.validate()
        return cfg

    def validate(self) -> None:
        if self.transformer != "hadamard":
            raise ValueError("the runtime only supports transformer='hadamard'")
        if self.codec != "ans":
            raise ValueError("the runtime only supports codec='ans' (run as the kvs-rze-v1 lossless stage)")
        if type(self.slot_count) is not int or self.slot_count < 1:
            raise ValueError("slot_count must be >= 1")
        if type(self.logical_blocks_per_chunk) is not int or self.logical_blocks_per_chunk < 1:
            raise ValueError("logical_blocks_per_chunk must be >= 1")
        stages = {"aggregate", "transformer", "quantizer", "codec"}
        unknown = set(self.pipeline) - stages
        if unknown:
            raise ValueError(f"Unknown compression stages: {sorted(unknown)}")
        if len(set(self.pipeline)) != len(self.pipeline):
            raise ValueError("compression stages must be unique")
        if "aggregate" not in self.pipeline:
            ordered = tuple(s for s in ("transformer", "quantizer", "codec") if s in self.pipeline)
            if self.pipeline != ordered:
                raise ValueError("compression stages must follow transformer, quantizer, codec order")
        elif len(self.pipeline) > 1:
            log.warning("the aggregate stage takes precedence over other compression stages")
        if not 0.0 <= self.hybrid_ratio <= 1.0:
            raise ValueError("hybrid_ratio must be in [0, 1]")
        for name in ("high_key_num_levels", "high_value_num_levels", "low_key_num_levels", "low_value_num_levels"):
            v = getattr(self, name)
            if type(v) is not int or not 2 <= v <= 256:
                raise ValueError(f"{name} must be an integer in [2, 256]")
        if self.split_type not in ("head", "layer"):
            raise ValueError(f"Unsupported split_type: {self.split_type}")
        if self.axis_key not in ("channel", "token", "tensor") or self.axis_value not in ("channel", "token", "tensor"):
            raise ValueError("unsupported quantization axis")
