"""Fixed-profile runtime configuration, parsed from a declarative schema.

``CompressionConfig.from_extra_config(extra)`` accepts the public keys of
kvserve_v1/compression/runtime/config.py:17-221 (``extra["compression"]`` with
the switch ``"enable-compression-pipeline"``, or the lossless aggregate
transport ``extra["raw_aggregate"]`` / ``extra["raw_agg"]``; the aggregate
transport wins when both are given).  Key names and defaults are the API and
stay as the reference publishes them; the parsing is one loop over
:data:`FIELDS`, a table that gives every key its kind, its allowed values or
range and its default, plus one whole-config rule (the pipeline's stage order).
"""
from __future__ import annotations

import logging
from dataclasses import dataclass, fields
from typing import Any, Literal, Optional

log = logging.getLogger("kvserve_b200.runtime")

STAGE_ORDER = ("transformer", "quantizer", "codec")
SWITCH = "enable-compression-pipeline"
AGGREGATE_KEYS = ("raw_aggregate", "raw_agg")


@dataclass(frozen=True)
class Field:
    """One configuration key: ``kind`` is int/float/str/choice/tuple."""
    kind: str
    default: Any
    lo: Optional[float] = None
    hi: Optional[float] = None
    choices: tuple = ()
    nullable: bool = False

    def coerce(self, key: str, value: Any) -> Any:
        if value is None and self.nullable:
            return None
        if self.kind == "int":
            if isinstance(value, bool) or not isinstance(value, int):
                raise ValueError(f"{key} must be an integer, got {value!r}")
        elif self.kind == "float":
            if isinstance(value, bool) or not isinstance(value, (int, float)):
                raise ValueError(f"{key} must be a number, got {value!r}")
            value = float(value)
        elif self.kind == "str":
            if not isinstance(value, str):
                raise ValueError(f"{key} must be a string, got {value!r}")
        elif self.kind == "choice":
            if value not in self.choices:
                raise ValueError(f"{key} must be one of {list(self.choices)}, got {value!r}")
        elif self.kind == "tuple":
            if isinstance(value, str) or not hasattr(value, "__iter__"):
                raise ValueError(f"{key} must be a list of stage names")
            value = tuple(value)
            bad = [s for s in value if s not in self.choices]
            if bad:
                raise ValueError(f"{key}: unknown stages {bad}; known {list(self.choices)}")
            if len(set(value)) != len(value):
                raise ValueError(f"{key}: stages must be unique")
        if self.lo is not None and not (self.lo <= value <= self.hi):
            raise ValueError(f"{key} must be in [{self.lo}, {self.hi}], got {value!r}")
        return value


# key -> schema; the defaults are the reference's published defaults
FIELDS: dict[str, Field] = {
    "transformer": Field("choice", "hadamard", choices=("hadamard",)),
    "seed": Field("int", 3237919422),
    "split_type": Field("choice", "layer", choices=("head", "layer")),
    "score_path": Field("str", None, nullable=True),
    "hybrid_ratio": Field("float", 0.8, 0.0, 1.0),
    "axis_key": Field("choice", "channel", choices=("channel", "token", "tensor")),
    "axis_value": Field("choice", "token", choices=("channel", "token", "tensor")),
    "high_key_num_levels": Field("int", 12, 2, 256),
    "high_value_num_levels": Field("int", 8, 2, 256),
    "low_key_num_levels": Field("int", 6, 2, 256),
    "low_value_num_levels": Field("int", 4, 2, 256),
    # "ans" names the lossless stage; it runs this project's kvs-rze-v1 codec
    "codec": Field("choice", "ans", choices=("ans",)),
    "slot_count": Field("int", 2, 1, 1 << 20),
    "logical_blocks_per_chunk": Field("int", 1, 1, 1 << 30),
    "pipeline": Field("tuple", STAGE_ORDER, choices=("aggregate",) + STAGE_ORDER),
}

# the aggregate transport's own keys (object form of raw_aggregate)
AGGREGATE_FIELDS: dict[str, Field] = {
    "slot_count": Field("int", 2, 1, 1 << 20),
    "logical_blocks_per_chunk": Field("int", 160, 1, 1 << 30),
}


def parse_fields(schema: dict[str, Field], raw: dict, where: str) -> dict:
    unknown = sorted(set(raw) - set(schema))
    if unknown:
        raise ValueError(f"{where}: unknown keys {unknown}")
    return {k: f.coerce(k, raw[k]) if k in raw else f.default for k, f in schema.items()}


def check_pipeline(stages: tuple) -> None:
    if "aggregate" in stages:
        if len(stages) > 1:
            log.warning("the aggregate stage takes precedence over other compression stages")
        return
    if stages != tuple(s for s in STAGE_ORDER if s in stages):
        raise ValueError(f"pipeline stages must appear in the order {list(STAGE_ORDER)}, got {list(stages)}")


@dataclass(frozen=True)
class CompressionConfig:
    enabled: bool = False
    transport: Literal["raw", "compression", "raw_aggregate"] = "compression"
    transformer: str = FIELDS["transformer"].default
    seed: int = FIELDS["seed"].default
    split_type: str = FIELDS["split_type"].default
    score_path: Optional[str] = None
    hybrid_ratio: float = FIELDS["hybrid_ratio"].default
    axis_key: str = FIELDS["axis_key"].default
    axis_value: str = FIELDS["axis_value"].default
    high_key_num_levels: int = FIELDS["high_key_num_levels"].default
    high_value_num_levels: int = FIELDS["high_value_num_levels"].default
    low_key_num_levels: int = FIELDS["low_key_num_levels"].default
    low_value_num_levels: int = FIELDS["low_value_num_levels"].default
    codec: str = FIELDS["codec"].default
    slot_count: int = FIELDS["slot_count"].default
    logical_blocks_per_chunk: int = FIELDS["logical_blocks_per_chunk"].default
    pipeline: tuple = STAGE_ORDER

    # ------------------------------------------------------------ queries
    @property
    def available(self) -> bool:
        return self.enabled

    @property
    def is_raw_aggregate(self) -> bool:
        return self.transport == "raw_aggregate"

    def uses(self, stage: str) -> bool:
        """Whether ``stage`` runs (the aggregate stage replaces all others)."""
        if stage == "aggregate":
            return "aggregate" in self.pipeline
        return "aggregate" not in self.pipeline and stage in self.pipeline

    uses_aggregate = property(lambda self: self.uses("aggregate"))
    uses_transformer = property(lambda self: self.uses("transformer"))
    uses_quantizer = property(lambda self: self.uses("quantizer"))
    uses_codec = property(lambda self: self.uses("codec"))

    # ------------------------------------------------------------ parsing
    @classmethod
    def from_extra_config(cls, extra_config: Optional[dict[str, Any]]) -> "CompressionConfig":
        extra = extra_config or {}
        comp = extra.get("compression") or {}
        agg_key = next((k for k in AGGREGATE_KEYS if k in extra), None)
        agg = extra.get(agg_key) if agg_key else None
        if agg not in (None, False):
            if agg is True:
                agg = {}
            if not isinstance(agg, dict):
                raise ValueError(f"{agg_key} must be true or an object with "
                                 f"{'/'.join(AGGREGATE_FIELDS)}")
            vals = parse_fields(AGGREGATE_FIELDS, agg, agg_key)
            if comp.get(SWITCH):
                log.warning("%s transport selected; compression keys %s are ignored", agg_key,
                            ", ".join(sorted(map(str, comp))))
            return cls(enabled=True, transport="raw_aggregate", pipeline=("aggregate",), **vals)
        if not comp.get(SWITCH, False):
            return cls(enabled=False, transport="raw")
        vals = parse_fields(FIELDS, {k: v for k, v in comp.items() if k != SWITCH}, "compression")
        cfg = cls(enabled=True, transport="compression", **vals)
        cfg.validate()
        return cfg

    def validate(self) -> None:
        """Re-check every field against the schema and the whole-config rules."""
        own = {f.name for f in fields(self)}
        for key, f in FIELDS.items():
            if key in own:
                f.coerce(key, getattr(self, key))
        check_pipeline(tuple(self.pipeline))
