"""Evaluators of the offline search (role of
kvserve_v1/offline_search/evaluation/param_search/{cr,acc}_evaluator.py).

* ``CompressionEvaluator`` — compression ratio of a configuration on a KV
  sample ``[L, 2, B, S, H, D]`` through the real modular pipeline (the same
  code the connector runs), cached per configuration in a CSV so a search
  can resume.
* ``AttentionFidelityEvaluator`` — a quality proxy for environments without
  an LM-eval harness: with random queries, the relative error of the
  attention outputs computed from the reconstructed KV versus the original,
  mapped to an "accuracy" in [0, 1] (1 - error).  Any callable
  ``config -> accuracy`` (e.g. an LM-eval run) can replace it.
"""
from __future__ import annotations

import csv
import json
import math
import os
from typing import Callable, Optional

import torch

from ..compression.adapter import KVCompressionAdapter


class CompressionEvaluator:
    def __init__(self, kv: torch.Tensor, num_kv_heads: int, head_size: int, cache_path: Optional[str] = None,
                 num_layers: Optional[int] = None):
        self.kv = kv
        self.H, self.D = num_kv_heads, head_size
        self.L = num_layers or kv.shape[0]
        self.cache_path = cache_path
        self._cache: dict[str, float] = {}
        if cache_path and os.path.exists(cache_path):
            with open(cache_path) as f:
                for row in csv.DictReader(f):
                    self._cache[row["config"]] = float(row["compression_ratio"])

    def _key(self, cfg: dict) -> str:
        return json.dumps(cfg, sort_keys=True)

    def evaluate(self, cfg: dict) -> tuple[float, Optional[torch.Tensor]]:
        key = self._key(cfg)
        ad = KVCompressionAdapter(cfg, self.H, self.D, num_layers=self.L)
        c = ad.compress(self.kv, "offline")
        if c is None:
            return 1.0, self.kv
        ratio = c.original_size / max(1, c.compressed_size)
        if key not in self._cache:
            self._cache[key] = ratio
            if self.cache_path:
                new = not os.path.exists(self.cache_path)
                with open(self.cache_path, "a", newline="") as f:
                    w = csv.DictWriter(f, fieldnames=["config", "compression_ratio"])
                    if new:
                        w.writeheader()
                    w.writerow({"config": key, "compression_ratio": ratio})
        return ratio, ad.decompress(c)

    def ratio(self, cfg: dict) -> float:
        key = self._key(cfg)
        if key in self._cache:
            return self._cache[key]
        return self.evaluate(cfg)[0]


class AttentionFidelityEvaluator:
    def __init__(self, kv: torch.Tensor, q_heads_per_kv: int = 4, num_queries: int = 32, seed: int = 0):
        self.kv = kv
        g = torch.Generator(device="cpu").manual_seed(seed)
        L, _, B, S, H, D = kv.shape
        # queries near real keys make the attention peaked, as in trained models
        keys = kv[:, 0].reshape(L, B * S, H, D).float().repeat_interleave(q_heads_per_kv, dim=2)
        pick = torch.randint(0, B * S, (num_queries,), generator=g)
        self.q = 2.0 * keys[:, pick] + 0.5 * torch.randn((L, num_queries, H * q_heads_per_kv, D), generator=g)
        self.group = q_heads_per_kv
        self._ref = self._attn(kv.float())

    def _attn(self, kv: torch.Tensor) -> torch.Tensor:
        L, _, B, S, H, D = kv.shape
        k = kv[:, 0].reshape(L, B * S, H, D).repeat_interleave(self.group, dim=2).to(self.q.device)
        v = kv[:, 1].reshape(L, B * S, H, D).repeat_interleave(self.group, dim=2).to(self.q.device)
        s = torch.einsum("lqhd,lthd->lhqt", self.q, k.float()) / math.sqrt(D)
        return torch.einsum("lhqt,lthd->lqhd", s.softmax(-1), v.float())

    def accuracy(self, reconstructed: torch.Tensor) -> float:
        out = self._attn(reconstructed.float().cpu())
        err = ((out - self._ref).norm() / self._ref.norm().clamp_min(1e-12)).item()
        return max(0.0, 1.0 - err)


def speed_model(cfg: dict, hbm_gbps: float = 6458.4) -> float:
    """Harmonic encode/decode speed (MB/s) of a profile on the fused path:
    both directions are memory-bound single passes (read bf16 KV + write the
    packed stream), so S ~ HBM bandwidth / (bytes touched per input byte)."""
    per_byte = 1.0 + 0.5  # read input once, write <= half as packed symbols (upper bound)
    s1 = s2 = hbm_gbps * 1e3 / per_byte
    return s1 * s2 / (s1 + s2)
