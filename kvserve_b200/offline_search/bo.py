"""Constraint-aware Bayesian optimisation over compression profiles (method of
kvserve_v1/offline_search/evaluation/param_search/test_search.py:237-604):
a Gaussian process (Matern nu=1.5 + white noise) predicts accuracy from the
point's features; the acquisition maximises the compression ratio weighted by
the probability of meeting the accuracy threshold plus an exploration bonus
``w * sigma * mean(cr)``; measured points prune dominated ones (monotonic
precision); the search stops after ``patience`` rounds without improvement.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Callable, Optional

import numpy as np

from .space import SearchPoint


@dataclass
class Observation:
    point: SearchPoint
    compression_ratio: float
    accuracy: float


@dataclass
class SearchResult:
    best: Optional[Observation]
    observations: list = field(default_factory=list)
    pruned: int = 0


def _normal_cdf(z: np.ndarray) -> np.ndarray:
    return 0.5 * (1.0 + np.vectorize(math.erf)(z / math.sqrt(2.0)))


class ConstraintAwareBO:
    def __init__(self, threshold: float, explore_weight: float = 0.1, seed: int = 0):
        self.threshold = threshold
        self.w = explore_weight
        self.rng = np.random.default_rng(seed)
        self.gp = None

    def fit(self, obs: list[Observation]) -> None:
        from sklearn.gaussian_process import GaussianProcessRegressor
        from sklearn.gaussian_process.kernels import Matern, WhiteKernel
        X = np.array([o.point.features() for o in obs])
        y = np.array([o.accuracy for o in obs])
        self.gp = GaussianProcessRegressor(kernel=Matern(nu=1.5) + WhiteKernel(1e-4), normalize_y=True,
                                           random_state=0)
        self.gp.fit(X, y)

    def propose(self, candidates: list[SearchPoint], ratios: dict) -> Optional[SearchPoint]:
        if not candidates:
            return None
        X = np.array([c.features() for c in candidates])
        mu, sd = self.gp.predict(X, return_std=True)
        cr = np.array([ratios[c] for c in candidates])
        p_ok = _normal_cdf((mu - self.threshold) / np.maximum(sd, 1e-9))
        score = cr * p_ok + self.w * sd * cr.mean()
        return candidates[int(np.argmax(score))]


def search(points: list[SearchPoint], ratio_fn: Callable[[SearchPoint], float],
           accuracy_fn: Callable[[SearchPoint], float], threshold: float, budget: int = 20, seeds: int = 4,
           patience: int = 6, seed: int = 0) -> SearchResult:
    """Maximise compression ratio subject to accuracy >= threshold."""
    rng = np.random.default_rng(seed)
    ratios = {p: ratio_fn(p) for p in points}
    remaining = sorted(points, key=lambda p: -ratios[p])
    obs: list[Observation] = []
    infeasible: list[SearchPoint] = []
    feasible: list[SearchPoint] = []
    pruned = 0

    def measure(p: SearchPoint) -> None:
        nonlocal pruned
        acc = accuracy_fn(p)
        obs.append(Observation(p, ratios[p], acc))
        (feasible if acc >= threshold else infeasible).append(p)
        before = len(remaining)
        keep = []
        for q in remaining:
            if q == p:
                continue
            # a point with no more precision than an infeasible one is infeasible;
            # one with no less precision than a feasible point cannot beat its ratio much
            if acc < threshold and p.dominates_quality(q):
                continue
            keep.append(q)
        remaining[:] = keep
        pruned += before - len(remaining) - 1

    # seeds: the highest-ratio point plus random picks
    init = [remaining[0]] + list(rng.choice(remaining[1:], size=min(seeds - 1, len(remaining) - 1), replace=False)) \
        if len(remaining) > 1 else list(remaining)
    for p in init:
        if p in remaining:
            measure(p)
    bo = ConstraintAwareBO(threshold, seed=seed)
    best_ratio, stale = -1.0, 0
    while remaining and len(obs) < budget and stale < patience:
        bo.fit(obs)
        nxt = bo.propose(remaining, ratios)
        if nxt is None:
            break
        measure(nxt)
        cur = max((o.compression_ratio for o in obs if o.accuracy >= threshold), default=-1.0)
        stale = stale + 1 if cur <= best_ratio else 0
        best_ratio = max(best_ratio, cur)
    best = max((o for o in obs if o.accuracy >= threshold), key=lambda o: o.compression_ratio, default=None)
    return SearchResult(best, obs, pruned)
