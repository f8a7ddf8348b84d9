"""Search space of the offline profile search (role of
kvserve_v1/offline_search/evaluation/param_search/test_search.py:24-146).

A point is a modular-pipeline configuration: Hadamard on/off, hybrid ratio,
the four ``*_max_value`` levels and the lossless codec.  Validity and the
monotonic pruning relations (more levels / fewer low heads never lowers
accuracy) are what the Bayesian search uses to skip points.
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass
from typing import Iterable

LEVELS = (16, 12, 8, 6, 4)
RATIOS = (0.0, 0.2, 0.4, 0.6, 0.8, 1.0)


@dataclass(frozen=True)
class SearchPoint:
    hadamard: bool
    hybrid_ratio: float
    high_key: int
    high_value: int
    low_key: int
    low_value: int
    codec: str = "lc"

    def is_valid(self) -> bool:
        return self.low_key <= self.high_key and self.low_value <= self.high_value

    def dominates_quality(self, other: "SearchPoint") -> bool:
        """True if self keeps at least as much precision as ``other`` everywhere
        (so its accuracy is >= other's under the monotonicity assumption)."""
        return (self.hadamard == other.hadamard and self.codec == other.codec
                and self.hybrid_ratio <= other.hybrid_ratio and self.high_key >= other.high_key
                and self.high_value >= other.high_value and self.low_key >= other.low_key
                and self.low_value >= other.low_value)

    def features(self) -> list[float]:
        return [float(self.hadamard), self.hybrid_ratio, self.high_key / 16, self.high_value / 16,
                self.low_key / 16, self.low_value / 16]

    def to_config(self, model_name: str = "Llama-3.1-8B-Instruct", split_type: str = "head") -> dict:
        pipeline = (["transformer"] if self.hadamard else []) + ["quantizer", "codec"]
        cfg = {"enabled": True, "pipeline": pipeline,
               "quantizer_config": {"model_name": model_name, "hybrid_ratio": self.hybrid_ratio,
                                    "high_key_max_value": self.high_key, "high_value_max_value": self.high_value,
                                    "low_key_max_value": self.low_key, "low_value_max_value": self.low_value,
                                    "axis_key": "channel", "axis_value": "token", "split_type": split_type},
               "codec_config": ({"codec_type": "lc", "lc_algorithm": "TUPL8_1 BIT_8 RZE_2"} if self.codec == "lc"
                                else {"codec_type": "bitpack",
                                      # inclusive clamp: symbol max_value itself can occur
                                      "bitpack_bits": max(self.high_key, self.high_value).bit_length()}),
               "min_compress_size": 1024}
        if self.hadamard:
            cfg["transformer_config"] = {"transform_type": "hadamard", "seed": 3237919422}
        return cfg

    def name(self) -> str:
        return (f"{'had' if self.hadamard else 'raw'}_hs{self.hybrid_ratio:g}_k{self.high_key}-{self.low_key}"
                f"_v{self.high_value}-{self.low_value}_{self.codec}")


def enumerate_space(levels: Iterable[int] = LEVELS, ratios: Iterable[float] = RATIOS,
                    hadamard: Iterable[bool] = (True, False), codecs: Iterable[str] = ("lc",)) -> list[SearchPoint]:
    pts = []
    for h, r, hk, hv, lk, lv, c in itertools.product(hadamard, ratios, levels, levels, levels, levels, codecs):
        p = SearchPoint(h, r, hk, hv, lk, lv, c)
        if not p.is_valid():
            continue
        if r == 0.0 and (lk != hk or lv != hv):
            continue  # no low heads: low levels are irrelevant, keep one representative
        if r == 1.0 and (hk != lk or hv != lv):
            continue  # no high heads
        pts.append(p)
    return pts
