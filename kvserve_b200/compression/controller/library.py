"""Profile library JSON (kvserve_v1/compression/controller/profile_library.py):

    {"library_metadata": {...},
     "accuracy_buckets": [{"bucket_id", "acc_range": [lo, hi],
                           "bandwidth_intervals": [{"interval_id", "x_range": [lo, hi] (x = 1/B),
                                                    "candidate_profile_ids": [...],
                                                    "model_optimal_profile_id": ...}],
                           "pareto_profiles": [<Profile dict>, ...]}]}

A bucket matches ``lo <= acc < hi`` (else the closest bucket); an interval
matches ``lo <= 1/B < hi`` (else the last, lowest-bandwidth interval).
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Optional

from .profile import Profile


class ProfileLibrary:
    def __init__(self, json_path: str | Path | None = None, data: Optional[dict] = None):
        if data is None:
            p = Path(json_path)
            if not p.exists():
                raise FileNotFoundError(f"Profile library not found: {json_path}")
            data = json.loads(p.read_text())
        self.metadata = data.get("library_metadata", {})
        self.accuracy_buckets: list[dict] = data.get("accuracy_buckets", [])
        self.profile_map: dict[str, Profile] = {}
        for b in self.accuracy_buckets:
            for pd in b.get("pareto_profiles", []):
                p = Profile.from_dict(pd)
                self.profile_map[p.profile_id] = p
        self._validate()

    def _validate(self) -> None:
        if not self.accuracy_buckets:
            raise ValueError("Profile library has no accuracy buckets")
        for b in self.accuracy_buckets:
            for key in ("bucket_id", "acc_range", "bandwidth_intervals"):
                if key not in b:
                    raise ValueError(f"Bucket missing '{key}'")

    def to_dict(self) -> dict:
        return {"library_metadata": self.metadata, "accuracy_buckets": self.accuracy_buckets}

    def find_bucket(self, acc_req: float) -> Optional[dict]:
        for b in self.accuracy_buckets:
            lo, hi = b["acc_range"]
            if lo <= acc_req < hi:
                return b
        if not self.accuracy_buckets:
            return None
        return min(self.accuracy_buckets,
                   key=lambda b: min(abs(b["acc_range"][0] - acc_req), abs(b["acc_range"][1] - acc_req)))

    def find_interval(self, bucket: dict, B_mbps: float) -> Optional[dict]:
        x = 1.0 / B_mbps
        ivs = bucket.get("bandwidth_intervals", [])
        for iv in ivs:
            lo, hi = iv["x_range"]
            if lo <= x < hi:
                return iv
        return ivs[-1] if ivs else None

    def get_profile(self, pid: str) -> Optional[Profile]:
        return self.profile_map.get(pid)

    def get_candidate_profiles(self, bucket: dict, interval: dict) -> list[Profile]:
        return [p for p in (self.get_profile(i) for i in interval.get("candidate_profile_ids", [])) if p is not None]

    def get_optimal_profile(self, bucket: dict, interval: dict) -> Optional[Profile]:
        pid = interval.get("model_optimal_profile_id")
        return self.get_profile(pid) if pid else None

    def get_all_profiles(self) -> list[Profile]:
        return list(self.profile_map.values())

    def get_num_profiles(self) -> int:
        return len(self.profile_map)

    def get_num_buckets(self) -> int:
        return len(self.accuracy_buckets)

    def get_bucket_info(self, bucket_id: int) -> Optional[dict]:
        return next((b for b in self.accuracy_buckets if b["bucket_id"] == bucket_id), None)

    def summary(self) -> str:
        n_iv = sum(len(b.get("bandwidth_intervals", [])) for b in self.accuracy_buckets)
        n_c = sum(len(iv.get("candidate_profile_ids", [])) for b in self.accuracy_buckets
                  for iv in b.get("bandwidth_intervals", []))
        return (f"ProfileLibrary(model={self.metadata.get('model_name', 'Unknown')}, profiles={self.get_num_profiles()}, "
                f"buckets={self.get_num_buckets()}, intervals={n_iv}, candidates={n_c})")

    def __repr__(self) -> str:
        return f"ProfileLibrary(profiles={self.get_num_profiles()}, buckets={self.get_num_buckets()})"
