"""Two-tier online profile selection
(kvserve_v1/compression/controller/online_controller.py:18-282).

Tier 1: accuracy bucket -> bandwidth interval (1/B) -> candidates ->
Theorem-1 filter.  Tier 2: ``T_eff = T_hat + delta_bar`` per candidate, SLO
filter, then epsilon-greedy (explore uniformly / exploit min T_eff).
``update(context, T_obs)`` feeds the observed latency back.  ``None`` means
"send uncompressed" and the context carries the reason.
"""
from __future__ import annotations

import random
from typing import Any, Optional

from .analytical import AnalyticalModel
from .bandit import BanditStateManager
from .library import ProfileLibrary
from .profile import Profile


class OnlineController:
    def __init__(self, profile_library: ProfileLibrary, epsilon: float = 0.1,
                 bandit_state: Optional[BanditStateManager] = None, alpha: float = 0.2,
                 transfer_model: str = "corrected", rng: Optional[random.Random] = None):
        self.library = profile_library
        self.epsilon = epsilon
        self.bandit = bandit_state or BanditStateManager(alpha=alpha)
        self.model = AnalyticalModel(transfer_model)
        self.rng = rng or random.Random()
        self.reset_statistics()

    def reset_statistics(self) -> None:
        self.total_decisions = self.exploit_count = self.explore_count = self.no_compression_count = 0

    def _none(self, ctx: dict) -> tuple[None, dict]:
        self.no_compression_count += 1
        return None, ctx

    def select_profile(self, V_bytes: float, B_mbps: float, T_model_ms: float, T_SLO_ms: float,
                       acc_req: float) -> tuple[Optional[Profile], dict[str, Any]]:
        self.total_decisions += 1
        bucket = self.library.find_bucket(acc_req)
        if bucket is None:
            return self._none({"reason": "no_matching_bucket", "acc_req": acc_req})
        interval = self.library.find_interval(bucket, B_mbps)
        if interval is None:
            return self._none({"reason": "no_matching_interval", "B_mbps": B_mbps})
        bid, iid = bucket["bucket_id"], interval["interval_id"]
        cands = self.library.get_candidate_profiles(bucket, interval)
        if not cands:
            return self._none({"reason": "no_candidates", "bucket_id": bid, "interval_id": iid})
        cands = [p for p in cands if self.model.check_benefit(p, B_mbps)]
        if not cands:
            return self._none({"reason": "no_benefit", "B_mbps": B_mbps, "bucket_id": bid, "interval_id": iid})
        base = self.model.predict_baseline_latency(V_bytes, B_mbps, T_model_ms)
        preds = {}
        for p in cands:
            t_hat = self.model.predict_latency(p, V_bytes, B_mbps, T_model_ms)
            _, d = self.bandit.get_stats(bid, iid, p.profile_id)
            t_eff = t_hat + d
            if t_eff <= T_SLO_ms:
                preds[p.profile_id] = {"profile": p, "T_hat": t_hat, "T_eff": t_eff, "delta_bar": d,
                                       "speedup": base / t_eff if t_eff > 0 else float("inf")}
        if not preds:
            return self._none({"reason": "slo_violation", "T_SLO_ms": T_SLO_ms, "bucket_id": bid,
                               "interval_id": iid, "candidates": [p.profile_id for p in cands]})
        if self.rng.random() < self.epsilon:
            action, pid = "explore", self.rng.choice(list(preds))
            self.explore_count += 1
        else:
            action, pid = "exploit", min(preds, key=lambda k: preds[k]["T_eff"])
            self.exploit_count += 1
        sel = preds[pid]
        return sel["profile"], {"bucket_id": bid, "interval_id": iid, "profile_id": pid, "T_hat": sel["T_hat"],
                                "T_eff": sel["T_eff"], "delta_bar": sel["delta_bar"],
                                "speedup_predicted": sel["speedup"], "action": action, "num_candidates": len(cands),
                                "baseline_latency": base, "V_bytes": V_bytes, "B_mbps": B_mbps,
                                "T_model_ms": T_model_ms, "T_SLO_ms": T_SLO_ms}

    def update(self, context: dict, T_obs_ms: float) -> None:
        if "profile_id" not in context:
            return
        self.bandit.update(context["bucket_id"], context["interval_id"], context["profile_id"],
                           T_obs_ms - context["T_hat"])

    def get_statistics(self) -> dict[str, Any]:
        n, ee = self.total_decisions, self.exploit_count + self.explore_count
        return {"total_decisions": n, "exploit_count": self.exploit_count, "explore_count": self.explore_count,
                "no_compression_count": self.no_compression_count,
                "compression_rate": (n - self.no_compression_count) / n if n else 0,
                "exploitation_rate": self.exploit_count / ee if ee else 0,
                "bandit_states": self.bandit.get_total_states(), "bandit_memory_bytes": self.bandit.get_memory_size()}

    def save_state(self, path: str) -> None:
        self.bandit.save(path)

    def load_state(self, path: str) -> None:
        self.bandit.load(path)
