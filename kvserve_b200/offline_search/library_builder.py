"""Assemble a controller profile library from measured profiles.

The reference consumes this JSON (kvserve_v1/compression/controller/
profile_library.py:17-171) but ships no code that produces it.  Here:

* accuracy buckets are consecutive ``[lo, hi)`` ranges; a bucket's Pareto set
  is every profile whose accuracy reaches ``lo`` and that no other such
  profile beats on both compression ratio and codec speed;
* in x = 1/B space the predicted latency of a profile is affine,
  ``T_p(x) = V/S + V x / cr`` (and ``T_0(x) = V x`` uncompressed); the lower
  envelope over the Pareto set splits the x axis into intervals, each with
  its optimal profile (Theorem 2); the candidate list of an interval is that
  optimum plus its envelope neighbours (2-3 profiles);
* profiles never beneficial anywhere in an interval (Theorem 1) are dropped.
"""
from __future__ import annotations

import json
from typing import Iterable, Optional

from ..compression.controller.profile import Profile


def _pareto(profiles: list[Profile]) -> list[Profile]:
    out = []
    for p in profiles:
        dominated = any(q is not p and q.compression_ratio >= p.compression_ratio and q.harmonic_speed >= p.harmonic_speed
                        and (q.compression_ratio > p.compression_ratio or q.harmonic_speed > p.harmonic_speed)
                        for q in profiles)
        if not dominated:
            out.append(p)
    return out


def _envelope(profiles: list[Profile], x_max: float, samples: int = 4096) -> list[tuple[float, float, Optional[Profile]]]:
    """Piecewise-optimal choice over x in [0, x_max] (None = no compression)."""
    segs: list[tuple[float, float, Optional[Profile]]] = []
    prev, start = "unset", 0.0
    for i in range(samples + 1):
        x = x_max * i / samples
        best, best_t = None, x  # per MB of KV: uncompressed costs x (ms per MB scaled)
        for p in profiles:
            t = 1.0 / p.harmonic_speed + x / p.compression_ratio
            if t < best_t:
                best, best_t = p, t
        if prev == "unset":
            prev = best
        elif best is not prev:
            segs.append((start, x, prev))
            start, prev = x, best
    segs.append((start, float("inf"), prev))
    return segs


def build_library(profiles: Iterable[Profile], acc_edges: list[float], b_min_mbps: float = 10.0,
                  model_name: str = "", dataset: str = "synthetic") -> dict:
    profiles = list(profiles)
    x_max = 1.0 / b_min_mbps
    buckets = []
    for bid, (lo, hi) in enumerate(zip(acc_edges[:-1], acc_edges[1:])):
        eligible = [p for p in profiles if p.accuracy >= lo]
        pareto = _pareto(eligible)
        segs = _envelope(pareto, x_max)
        ordered = [s[2] for s in segs]
        intervals = []
        for iid, (x0, x1, opt) in enumerate(segs):
            cands = []
            for k in (iid - 1, iid, iid + 1):
                if 0 <= k < len(ordered) and ordered[k] is not None and ordered[k].profile_id not in cands:
                    cands.append(ordered[k].profile_id)
            intervals.append({"interval_id": iid, "x_range": [x0, x1 if x1 != float("inf") else 1e30],
                              "candidate_profile_ids": cands,
                              "model_optimal_profile_id": opt.profile_id if opt else None})
        buckets.append({"bucket_id": bid, "acc_range": [lo, hi], "bandwidth_intervals": intervals,
                        "pareto_profiles": [p.to_dict() for p in pareto]})
    return {"library_metadata": {"model_name": model_name, "dataset": dataset, "num_profiles": len(profiles)},
            "accuracy_buckets": buckets}


def save_library(lib: dict, path: str) -> None:
    with open(path, "w") as f:
        json.dump(lib, f, indent=2)
