"""Service-aware PD serving: the online controller picks the KV transfer
profile of every request (roles of kvserve_v1/compression/controller/online_controller.py:18-282
and the adapter's controller mode, kvserve_v1/compression/adapter.py).

    python -m torch.distributed.run --nnodes 1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        --master-port P -m kvserve_b200.engine.serving --model llama-3-70b --prompt-len 16384 \\
        --max-new 256 --rate 1.0 --link-gbps 25,100,400 --requests 8

The engine holds every profile of :data:`ENGINE_PROFILES` (8-, 4-, 2-bit and
uncompressed); their compression ratios come from the engine's own frame
geometry, their codec speeds from the measured fused kernels (or an HBM
model) and their accuracy from an attention-fidelity proxy on synthetic KV
shaped like the benchmark's (values N(0,1); keys N(0,1) with 4 outlier
channels per head scaled x8).  A profile library is built from them
(:func:`~kvserve_b200.offline_search.library_builder.build_library`), and
for each request rank 0 asks :class:`OnlineController` for a profile given
the request's KV bytes, the emulated link bandwidth, the predicted prefill
time and the SLO, and broadcasts the choice; all ranks serve the request with
that profile with the encode kernels pacing their stores at the link cap.
The observed KV-ready time (max over ranks) feeds the controller's bandit.

Arrivals are a seeded Poisson process on a virtual clock: request i arrives
at a_i, starts at max(a_i, end of request i-1) and its queueing delay is
added to its TTFT, so no GPU time is spent sleeping.
"""
from __future__ import annotations

import argparse
import json
import math
import random
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.distributed as dist

from .transfer import TransferProfile

# "off" is the uncompressed transfer the controller falls back to (None).
ENGINE_PROFILES: dict[str, TransferProfile] = {
    "k8v8": TransferProfile(compressed=True, hybrid_ratio=0.0, key_levels=(256, 256), value_levels=(256, 256)),
    "k4v4": TransferProfile(compressed=True, hybrid_ratio=0.0, key_levels=(16, 16), value_levels=(16, 16)),
    "k4v2": TransferProfile(compressed=True, hybrid_ratio=0.0, key_levels=(16, 16), value_levels=(4, 4)),
    "k2v2": TransferProfile(compressed=True, hybrid_ratio=0.0, key_levels=(4, 4), value_levels=(4, 4)),
    "off": TransferProfile.raw(),
}


def synthetic_kv(tokens: int, heads: int, dim: int, seed: int = 0, outliers: int = 4) -> torch.Tensor:
    """``[1, 2, 1, tokens, heads, dim]`` bf16 KV: values N(0,1), keys N(0,1)
    with ``outliers`` fixed channels per head scaled x8."""
    g = torch.Generator().manual_seed(seed)
    kv = torch.randn((1, 2, 1, tokens, heads, dim), generator=g)
    ch = torch.randperm(dim, generator=g)[:outliers]
    kv[:, 0, ..., ch] *= 8.0
    return kv.to(torch.bfloat16)


def profile_accuracy(profile: TransferProfile, heads: int, dim: int, tokens: int = 256, seed: int = 0) -> float:
    """1 - relative error of attention outputs over the reconstructed KV
    (CPU frame oracle, the same arithmetic as the fused kernels)."""
    from ..compression.heads import rademacher_signs
    from ..offline_search.evaluators import AttentionFidelityEvaluator
    from ..ops import kv_codec as kc
    kv = synthetic_kv(tokens, heads, dim, seed)
    if not profile.compressed:
        return 1.0
    spec = kc.spec_from_profile(tokens, heads, dim, 0, profile.key_levels, profile.value_levels)
    order = torch.arange(heads, dtype=torch.int32)
    signs = rademacher_signs(profile.seed, 0, heads, dim)
    buf = kc.cpu_encode_frame(kv[0, 0, 0], kv[0, 1, 0], spec, order, signs)
    k, v = kc.cpu_decode_frame(bytes(buf), spec, order, signs)
    rec = torch.stack([k, v]).unsqueeze(0).unsqueeze(2)
    return AttentionFidelityEvaluator(kv).accuracy(rec)


def engine_library(engine, tokens: int, speeds_mbps: Optional[dict] = None,
                   acc_edges: Optional[tuple] = None) -> "ProfileLibrary":  # noqa: F821
    """Profile library of the engine's compressed profiles at ``tokens``.
    By default the accuracy buckets start at the profiles' own accuracies,
    so a bucket's lower edge is a quality every profile in it meets (use
    :func:`bucket_requirement` to map a requirement onto that edge)."""
    from ..compression.controller.library import ProfileLibrary
    from ..compression.controller.profile import Profile
    from ..offline_search.evaluators import speed_model
    from ..offline_search.library_builder import build_library
    profiles = []
    for name, x in engine.xfers.items():
        if not x.profile.compressed:
            continue
        cr = x.raw_bytes(tokens) / x.payload_bytes(tokens)
        s = (speeds_mbps or {}).get(name) or speed_model({})
        profiles.append(Profile(name, {"engine_profile": name}, x.profile.to_compression() or {},
                                {"compression_ratio": cr, "harmonic_speed_mbps": s},
                                {"accuracy": profile_accuracy(x.profile, x.H, x.D)}))
    if acc_edges is None:
        acc_edges = tuple([0.0] + sorted({p.accuracy for p in profiles}) + [1.01])
    return ProfileLibrary(data=build_library(profiles, list(acc_edges), model_name=engine.cfg.name))


def bucket_requirement(library, acc_req: float) -> Optional[float]:
    """The lowest bucket edge >= ``acc_req`` (None: no compressed profile is
    accurate enough, the request goes uncompressed)."""
    edges = sorted(b["acc_range"][0] for b in library.accuracy_buckets)
    ok = [e for e in edges if e >= acc_req]
    return ok[0] if ok else None


@dataclass
class ServedRequest:
    index: int
    link_gbps: float
    profile: str
    arrival_ms: float
    queue_ms: float
    ttft_ms: float          # queueing + first token (max over ranks)
    kv_ready_ms: float      # KV of the prompt in the decode rank's paged cache (max over ranks)
    request_ms: float
    payload_bytes: int
    decision: dict = field(default_factory=dict)


class ServiceAwareServer:
    """Drives a :class:`PDEngine` built with :data:`ENGINE_PROFILES`.  Every
    rank calls :meth:`serve` with the same arguments."""

    def __init__(self, engine, library, slo_ms: float, acc_req: float = 0.97, epsilon: float = 0.1,
                 seed: int = 0):
        from ..compression.controller.online import OnlineController
        self.engine = engine
        self.ctx = engine.ctx
        self.controller = OnlineController(library, epsilon=epsilon, rng=random.Random(seed))
        self.slo_ms, self.acc_req = slo_ms, acc_req
        self.t_model_ms: Optional[float] = None

    def _bcast(self, obj):
        if not self.ctx.distributed:
            return obj
        box = [obj]
        dist.broadcast_object_list(box, src=self.ctx.rank_offset, group=self.ctx.cpu_group)
        return box[0]

    def _max(self, vals: list[float]) -> list[float]:
        if not self.ctx.distributed:
            return vals
        t = torch.tensor([v if math.isfinite(v) else -1.0 for v in vals], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.ctx.cpu_group)
        return t.tolist()

    def serve(self, prompts: list[torch.Tensor], rate_per_s: float, link_gbps: float, max_new: int,
              seed: int = 0) -> list[ServedRequest]:
        rng = random.Random(seed)
        clock = 0.0
        free_at = 0.0
        out = []
        for i, p in enumerate(prompts):
            clock += rng.expovariate(rate_per_s) * 1e3 if rate_per_s > 0 else 0.0
            start = max(clock, free_at)
            decision = None
            if self.ctx.rank == 0:
                V = self.engine.xfer.raw_bytes(int(p.numel()))
                need = bucket_requirement(self.controller.library, self.acc_req)
                if need is None:
                    prof, info = None, {"reason": "accuracy", "acc_req": self.acc_req}
                else:
                    prof, info = self.controller.select_profile(V, link_gbps * 125.0, self.t_model_ms or 0.0,
                                                                self.slo_ms, need)
                decision = {"profile": prof.profile_id if prof is not None else "off", "info": info}
            decision = self._bcast(decision)
            res = self.engine.generate(p, max_new, profile=decision["profile"], link_gbps=link_gbps)
            t = res.timing
            first, kv_ready, prefill, total = self._max([t.first_token, t.ingest_done, t.prefill_done,
                                                          t.request_host])
            self.t_model_ms = prefill if self.t_model_ms is None else 0.8 * self.t_model_ms + 0.2 * prefill
            if self.ctx.rank == 0:
                self.controller.update(decision["info"], kv_ready)
            free_at = start + total
            out.append(ServedRequest(i, link_gbps, decision["profile"], clock, start - clock, start - clock + first,
                                     kv_ready, total, t.payload_bytes,
                                     {k: v for k, v in decision["info"].items() if isinstance(v, (int, float, str))}))
        return out


def _p50(xs: list[float]) -> float:
    s = sorted(xs)
    return s[len(s) // 2] if s else float("nan")


def _pct(xs: list[float], q: float) -> float:
    s = sorted(x for x in xs if x == x)
    return s[min(len(s) - 1, int(q * len(s)))] if s else float("nan")


def serve_pipelined(engine, library, prompts: list, rate_per_s: float, link_gbps: float, max_new: int, slo_ms: float,
                    acc_req: float, t_model_ms: float, max_batch: int = 8, seed: int = 0, server=None) -> dict:
    """Real-time Poisson arrivals on the pipelined server (prefill of one
    request overlaps the decode of earlier ones); the prefill leader's
    controller picks each request's profile and learns from the decode
    leader's KV-ready times.  Returns the summary of this link cap (every
    rank calls it; the summary is the same on all ranks)."""
    from ..compression.controller.online import OnlineController
    from .pipeline import PipelinedServer, Request, merge_records, poisson_schedule
    ctx = engine.ctx
    server = server or PipelinedServer(engine, max_batch=max_batch)
    ctrl = OnlineController(library, epsilon=0.1, rng=random.Random(seed))
    infos: dict[int, dict] = {}
    arrivals = poisson_schedule(len(prompts), rate_per_s, seed)
    reqs = [Request(i, p, max_new, a, link_gbps=link_gbps) for i, (p, a) in enumerate(zip(prompts, arrivals))]
    t_model = [t_model_ms]

    def decide(req, state):
        if state["prefill_ms"]:
            t_model[0] = 0.8 * t_model[0] + 0.2 * state["prefill_ms"][-1]
        V = engine.xfer.raw_bytes(int(req.prompt.numel()))
        need = bucket_requirement(library, acc_req)
        if need is None:
            infos[req.index] = {"reason": "accuracy"}
            return "off"
        prof, info = ctrl.select_profile(V, link_gbps * 125.0, t_model[0], slo_ms, need)
        infos[req.index] = info
        return prof.profile_id if prof is not None else "off"

    def feedback(req, kv_ready_ms):
        info = infos.get(req.index)
        if info is not None and "reason" not in info:
            ctrl.update(info, kv_ready_ms)

    recs = merge_records(ctx, server.serve(reqs, decide, feedback))
    span_s = max(r.done_ms + r.arrival_ms for r in recs) / 1e3
    counts: dict[str, int] = {}
    for r in recs:
        counts[r.profile] = counts.get(r.profile, 0) + 1
    return {"requests": len(recs), "rate_per_s": rate_per_s, "link_gbps": link_gbps,
            "ttft_ms_p50": round(_pct([r.first_token_ms for r in recs], 0.5), 3),
            "ttft_ms_p90": round(_pct([r.first_token_ms for r in recs], 0.9), 3),
            "queue_ms_p50": round(_pct([r.launch_ms for r in recs], 0.5), 3),
            "prefill_ms_p50": round(_pct([r.prefill_ms - r.launch_ms for r in recs], 0.5), 3),
            "request_ms_p50": round(_pct([r.done_ms for r in recs], 0.5), 3),
            "output_tokens_per_s": round(sum(len(r.tokens or []) for r in recs) / span_s, 2),
            "profiles": counts}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-70b")
    ap.add_argument("--prompt-len", type=int, default=16384)
    ap.add_argument("--max-new", type=int, default=256)
    ap.add_argument("--rate", type=float, default=1.0, help="Poisson arrivals per second")
    ap.add_argument("--link-gbps", default="25,100,400")
    ap.add_argument("--requests", type=int, default=8)
    ap.add_argument("--slo-ms", type=float, default=0.0, help="SLO on KV-ready time (0: 4x the first prefill)")
    ap.add_argument("--acc-req", type=float, default=0.97)
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (smoke runs)")
    ap.add_argument("--speeds", default="", help="JSON {profile: harmonic MB/s} measured by the microbench")
    ap.add_argument("--serial", action="store_true",
                    help="one request at a time on a virtual clock (default: pipelined, real-time arrivals)")
    ap.add_argument("--max-batch", type=int, default=8, help="decode rows of the pipelined server")
    a = ap.parse_args(argv)
    from ..models.config import get_config
    from ..parallel.context import destroy_parallel, init_parallel
    from .pd import PDEngine
    ctx = init_parallel("nccl", timeout_s=300)
    cfg = get_config(a.model)
    if a.layers:
        import dataclasses
        cfg = dataclasses.replace(cfg, num_layers=a.layers)
    engine = PDEngine(cfg, ctx, ENGINE_PROFILES["off"], max_prompt=a.prompt_len, max_new_tokens=a.max_new,
                      profiles=dict(ENGINE_PROFILES), max_batch=1 if a.serial else a.max_batch)
    engine.warmup(prompt_len=min(512, a.prompt_len))
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab, (a.prompt_len,), generator=g, dtype=torch.int32).pin_memory()
               for _ in range(a.requests)]
    library = engine_library(engine, a.prompt_len, json.loads(a.speeds) if a.speeds else None)
    # the first request calibrates the model-time estimate and the default SLO
    probe = engine.generate(prompts[0], 1, profile="k4v2")
    slo = a.slo_ms or 4.0 * probe.timing.prefill_done
    report = {"model": cfg.name, "prompt_len": a.prompt_len, "max_new": a.max_new, "rate_per_s": a.rate,
              "world": ctx.world_size, "slo_ms": round(slo, 2), "acc_req": a.acc_req,
              "library": [{"id": p.profile_id, "cr": round(p.compression_ratio, 3), "acc": round(p.accuracy, 4)}
                          for p in library.get_all_profiles()], "links": {}}
    report["mode"] = "serial (virtual clock)" if a.serial else f"pipelined (real-time arrivals, {a.max_batch} rows)"
    pserver = None
    if not a.serial:
        from .pipeline import PipelinedServer
        pserver = PipelinedServer(engine, max_batch=a.max_batch)
    for cap in (float(x) for x in a.link_gbps.split(",") if x):
        if pserver is not None:
            report["links"][f"{cap:g}"] = serve_pipelined(engine, library, prompts, a.rate, cap, a.max_new, slo,
                                                          a.acc_req, probe.timing.prefill_done, a.max_batch,
                                                          server=pserver)
            continue
        server = ServiceAwareServer(engine, library, slo, a.acc_req)
        server.t_model_ms = probe.timing.prefill_done
        served = server.serve(prompts, a.rate, cap, a.max_new)
        counts: dict[str, int] = {}
        for r in served:
            counts[r.profile] = counts.get(r.profile, 0) + 1
        report["links"][f"{cap:g}"] = {
            "ttft_ms_p50": round(_p50([r.ttft_ms for r in served]), 3),
            "kv_ready_ms_p50": round(_p50([r.kv_ready_ms for r in served]), 3),
            "queue_ms_p50": round(_p50([r.queue_ms for r in served]), 3),
            "request_ms_p50": round(_p50([r.request_ms for r in served]), 3),
            "profiles": counts,
            "controller": server.controller.get_statistics() if ctx.rank == 0 else None,
        }
    if ctx.rank == 0:
        print(json.dumps(report))
    torch.cuda.synchronize()
    engine.close()
    destroy_parallel(ctx)


if __name__ == "__main__":
    main()
