"""A compression profile: a pipeline config plus its measured compression
ratio, harmonic codec speed and accuracy
(kvserve_v1/compression/controller/profile.py:10-87)."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any


@dataclass
class Profile:
    profile_id: str
    metadata: dict = field(default_factory=dict)
    compression_config: dict = field(default_factory=dict)
    performance_metrics: dict = field(default_factory=dict)
    quality_metrics: dict = field(default_factory=dict)

    @classmethod
    def from_dict(cls, d: dict) -> "Profile":
        return cls(d["profile_id"], d.get("metadata", {}), d["compression_config"], d["performance_metrics"],
                   d["quality_metrics"])

    def to_dict(self) -> dict[str, Any]:
        return {"profile_id": self.profile_id, "metadata": self.metadata,
                "compression_config": self.compression_config, "performance_metrics": self.performance_metrics,
                "quality_metrics": self.quality_metrics}

    @property
    def compression_ratio(self) -> float:
        return float(self.performance_metrics["compression_ratio"])

    @property
    def harmonic_speed(self) -> float:
        """Harmonic encode/decode speed S = S1*S2/(S1+S2) in MB/s."""
        return float(self.performance_metrics["harmonic_speed_mbps"])

    @property
    def critical_bandwidth(self) -> float:
        """B_crit = (1 - 1/cr) * S: compression pays off below this bandwidth."""
        return float(self.performance_metrics.get("critical_bandwidth_mbps",
                                                  (1.0 - 1.0 / self.compression_ratio) * self.harmonic_speed))

    @property
    def accuracy(self) -> float:
        return float(self.quality_metrics["accuracy"])

    def __repr__(self) -> str:
        return f"Profile(id={self.profile_id}, cr={self.compression_ratio:.2f}, acc={self.accuracy:.3f})"
