"""Offline profile search driver (role of
kvserve_v1/offline_search/evaluation/param_search/test_search.py:main).

Phase 1 measures the compression ratio of every point of the search space
on a KV sample (cached in a CSV, so the search resumes).  Phase 2 runs the
constraint-aware Bayesian search for each accuracy tolerance.  Phase 3
turns the measured profiles into a controller profile library.

    python -m kvserve_b200.offline_search.search --out results/ \
        [--kv kv.pt] [--tolerances 1 3 5] [--budget 24] [--accuracy model]

Without ``--kv`` a synthetic sample with outlier key channels is used.  The
quality metric is the attention-fidelity proxy on the sample, or with
``--accuracy model`` the language-model evaluator of
:mod:`kvserve_b200.offline_search.model_eval` (a local checkpoint given by
``--hf-model``, else a random-init tiny Llama; its score in percent of the
default cache, as a fraction).
"""
from __future__ import annotations

import argparse
import json
import os
from typing import Optional

import torch

from ..compression.controller.profile import Profile
from .bo import search
from .evaluators import AttentionFidelityEvaluator, CompressionEvaluator, speed_model
from .library_builder import build_library, save_library
from .space import enumerate_space


def synthetic_kv(layers: int = 4, tokens: int = 512, heads: int = 8, dim: int = 128, seed: int = 0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    kv = torch.randn((layers, 2, 1, tokens, heads, dim), generator=g)
    ch = torch.randperm(dim, generator=g)[:4]
    kv[:, 0, :, :, :, ch] *= 8
    return kv.to(torch.bfloat16)


def run(out_dir: str, kv: Optional[torch.Tensor] = None, tolerances=(1.0, 3.0, 5.0), budget: int = 24,
        model_name: str = "synthetic", levels=(16, 12, 8, 6, 4), ratios=(0.0, 0.4, 0.8, 1.0),
        model_accuracy=None) -> dict:
    """``model_accuracy``: optional ``profile -> percent`` (e.g.
    :meth:`ModelAccuracyEvaluator.evaluate`) used instead of the
    attention-fidelity proxy."""
    os.makedirs(out_dir, exist_ok=True)
    kv = synthetic_kv() if kv is None else kv
    L, _, B, S, H, D = kv.shape
    comp = CompressionEvaluator(kv, H, D, cache_path=os.path.join(out_dir, "cr_cache.csv"), num_layers=L)
    fid = AttentionFidelityEvaluator(kv)
    points = enumerate_space(levels=levels, ratios=ratios)
    cfgs = {p: p.to_config(model_name) for p in points}
    for c in cfgs.values():
        c["quantizer_config"]["num_layers"] = L
        c["quantizer_config"]["num_kv_heads"] = H
    recon_cache: dict = {}

    def ratio(p):
        return comp.ratio(cfgs[p])

    def accuracy(p):
        if p not in recon_cache:
            if model_accuracy is not None:
                recon_cache[p] = model_accuracy(cfgs[p]) / 100.0
            else:
                _, rec = comp.evaluate(cfgs[p])
                recon_cache[p] = fid.accuracy(rec)
        return recon_cache[p]

    # accuracy tolerances are relative to the highest-precision point of the space
    ref = max(points, key=lambda p: (p.high_key + p.high_value + p.low_key + p.low_value, -p.hybrid_ratio,
                                     p.hadamard))
    baseline = accuracy(ref)
    results = {"baseline": {"name": ref.name(), "accuracy": baseline}}
    profiles = {}
    for tol in tolerances:
        thr = baseline - tol / 100.0
        res = search(points, ratio, accuracy, thr, budget=budget)
        results[str(tol)] = {
            "threshold": thr,
            "best": None if res.best is None else {"name": res.best.point.name(), "config": cfgs[res.best.point],
                                                   "compression_ratio": res.best.compression_ratio,
                                                   "accuracy": res.best.accuracy},
            "evaluated": len(res.observations), "pruned": res.pruned}
        for o in res.observations:
            profiles[o.point] = o
        with open(os.path.join(out_dir, f"tolerance_{tol:g}_results.json"), "w") as f:
            json.dump(results[str(tol)], f, indent=2)
    prof_objs = [Profile(o.point.name(), {"model_name": model_name}, cfgs[o.point],
                         {"compression_ratio": o.compression_ratio, "harmonic_speed_mbps": speed_model(cfgs[o.point])},
                         {"accuracy": o.accuracy}) for o in profiles.values()]
    lib = build_library(prof_objs, [0.0, 0.9, 0.95, 0.98, 1.01], model_name=model_name)
    save_library(lib, os.path.join(out_dir, "profile_library.json"))
    return {"results": results, "library": lib}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="offline_search_results")
    ap.add_argument("--kv", default=None, help="torch file with a [L, 2, B, S, H, D] KV sample")
    ap.add_argument("--tolerances", type=float, nargs="+", default=[1.0, 3.0, 5.0])
    ap.add_argument("--budget", type=int, default=24)
    ap.add_argument("--model-name", default="synthetic")
    ap.add_argument("--accuracy", choices=("fidelity", "model"), default="fidelity")
    ap.add_argument("--hf-model", default=None, help="local checkpoint for --accuracy model")
    args = ap.parse_args()
    kv = torch.load(args.kv) if args.kv else None
    model_accuracy = None
    if args.accuracy == "model":
        from .model_eval import ModelAccuracyEvaluator, synthetic_prompts, tiny_llama
        if args.hf_model:
            from transformers import AutoModelForCausalLM
            lm = AutoModelForCausalLM.from_pretrained(args.hf_model, torch_dtype=torch.float32).eval()
        else:
            lm = tiny_llama()
        ev = ModelAccuracyEvaluator(lm, synthetic_prompts(4, 256, lm.config.vocab_size))
        model_accuracy = ev.evaluate
    out = run(args.out, kv, tuple(args.tolerances), args.budget, args.model_name, model_accuracy=model_accuracy)
    print(json.dumps(out["results"], indent=2))


if __name__ == "__main__":
    main()
