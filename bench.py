"""Headline benchmark: TTFT p50 and KV-transfer ms per request of a
disaggregated prefill -> decode deployment (BASELINE.json metric).

Config: Llama-3.1-8B-shaped decoder, random-init
bf16 weights, 8192-token random prompts, 128 greedy output tokens, K 4-bit /
V 2-bit compressed KV hand-off.  N GPUs of one node:

* N = 1: prefill and decode colocated on one GPU (device-local hand-off);
* N = 2k: k prefill ranks (TP k) -> k decode ranks (TP k): 1P1D, 2P2D, 4P4D.

One step = one request end to end: prefill of the whole prompt, which
samples the first token; layer-streamed compressed KV push over NVLink; the
decode side continues from the first token with the remaining greedy tokens.
TTFT (max over ranks) is when both the first token exists and the decode
side holds the prompt's KV and that token, ready for the next step.  Timing: CUDA events per rank after a device-side
NCCL barrier, max over ranks; the prompt H2D copy (pinned) and the token D2H
copy are inside every step.  Inputs (8192 x 32 layers of KV, 16 GB of
weights) are far larger than L2, so no explicit flush is needed.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time

import torch

BASELINE_METRIC = "TTFT p50 + KV-transfer ms/request (max over ranks), 1P1D–4P4D on B200"


def _emit(obj) -> None:
    print(json.dumps(obj), flush=True)


def _log(msg: str) -> None:
    if os.environ.get("KVS_BENCH_VERBOSE"):
        print(f"[bench r{os.environ.get('RANK', '0')} {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def _profile(name: str):
    """``raw``, a named engine profile (k8v8, k4v4, k4v2, k2v2, off) or a
    ``configs/compression`` JSON file."""
    from kvserve_b200.engine.serving import ENGINE_PROFILES
    from kvserve_b200.engine.transfer import TransferProfile
    if name == "raw":
        return TransferProfile.raw()
    if name in ENGINE_PROFILES:
        return ENGINE_PROFILES[name]
    if os.path.exists(name):
        with open(name) as f:
            return TransferProfile.from_compression(json.load(f))
    raise SystemExit(f"unknown profile {name!r}")


def _handoff_roofline_ms(raw_bytes: int, payload_bytes: int, n_gpus: int) -> float:
    """Speed-of-light time of one rank pair's hand-off (bytes of one rank)."""
    hbm = 6650.0
    try:
        with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")) as f:
            hbm = float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        pass
    if n_gpus == 1:
        return 2 * (raw_bytes + payload_bytes) / (hbm * 1e6)
    return max((raw_bytes + payload_bytes) / (hbm * 1e6), payload_bytes / 770e6)


def run_reference(args) -> None:
    """The unmodified reference (baseline/_ref) through its own public API:
    vLLM V1 producer/consumer engines with its CompressedKVConnector."""
    from kvserve_b200.baselines.reference_arm import run
    args.metric = BASELINE_METRIC
    run(args, _emit)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--prompt-len", type=int, default=8192)
    ap.add_argument("--max-new", type=int, default=128)
    ap.add_argument("--profile", default="k4v2")
    ap.add_argument("--link-gbps", type=float, default=0.0)
    ap.add_argument("--layers", type=int, default=0, help="override layer count (smoke runs only)")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--ref-engine", default="vllm", choices=["vllm", "stock", "handoff"],
                    help="reference arm: 'vllm' (default) checks the stock stack once on a tiny model, then "
                         "serves the bench through vLLM with the reference connector under a vLLM-API adapter "
                         "and measures its KV hand-off alone; 'stock' only runs the stock check; 'handoff' only "
                         "measures the hand-off path (compression + NcclTransport) without vLLM")
    ap.add_argument("--ref-cuda-graphs", action="store_true",
                    help="reference arm: let vLLM capture CUDA graphs (default eager, as the reference's own PD "
                         "tests run; capture fails with its connector's per-layer save hook)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if os.environ.get("KVS_BENCH_DUMP_AFTER"):
        import faulthandler
        faulthandler.dump_traceback_later(float(os.environ["KVS_BENCH_DUMP_AFTER"]), repeat=True)

    from kvserve_b200.models.config import get_config
    from kvserve_b200.parallel.context import init_parallel, destroy_parallel
    from kvserve_b200.engine.pd import PDEngine
    from kvserve_b200.utils.clocks import ClockSampler
    import torch.distributed as dist

    ctx = init_parallel("nccl", timeout_s=300.0)
    if (ctx.job_world_size or ctx.world_size) != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={ctx.job_world_size or ctx.world_size}")
    n_rep = ctx.num_replicas   # data-parallel PD replicas (KVSERVE_REPLICAS), each of ctx.world_size GPUs
    cfg = get_config(args.model)
    if args.layers:
        cfg = cfg.with_layers(args.layers)
    profile = _profile(args.profile)
    engine = PDEngine(cfg, ctx, profile, max_prompt=args.prompt_len, max_new_tokens=args.max_new,
                      link_gbps=args.link_gbps, use_graphs=not args.no_graphs)
    _log("engine built")
    engine.warmup(prompt_len=min(512, args.prompt_len))
    _log("engine warm")

    g = torch.Generator().manual_seed(1234)
    prompts = [torch.randint(0, cfg.vocab, (args.prompt_len,), generator=g, dtype=torch.int32).pin_memory()
               for _ in range(args.warmup + args.steps)]
    for i in range(args.warmup):
        engine.generate(prompts[i], args.max_new)
        _log(f"warmup step {i} done")

    sampler = None
    if ctx.global_rank == 0:
        sampler = ClockSampler(list(range(torch.cuda.device_count())) if ctx.distributed else
                               [torch.cuda.current_device()])
        sampler.start()
    if ctx.distributed:
        dist.barrier(group=ctx.cpu_group)
    torch.cuda.synchronize()
    t_wall = time.perf_counter()
    timings = []
    for i in range(args.steps):
        res = engine.generate(prompts[args.warmup + i], args.max_new)
        timings.append(res.timing)
    torch.cuda.synchronize()
    if ctx.distributed:
        dist.barrier(group=ctx.cpu_group)
    wall_s = time.perf_counter() - t_wall
    clocks = sampler.stop() if sampler else None

    # the hand-off of one request on its own (no prefill beside it), and the
    # reconstruction error of the profile on synthetic KV; both after the
    # timed region
    handoffs = [engine.measure_handoff(args.prompt_len) for _ in range(3)]
    recon = None
    if ctx.rank == 0:
        from kvserve_b200.engine.fidelity import measure_profile
        recon = measure_profile(profile, min(4, cfg.num_layers), args.prompt_len, cfg.num_kv_heads, cfg.head_dim,
                                engine.device)

    # optional: per-kernel device time of a decode step (profiler; not a
    # timing of record), the table the N=8 scaling analysis needs
    ktable = None
    if os.environ.get("KVSERVE_PROFILE_DECODE", "1") != "0":
        try:
            ktable = engine.decode_kernel_table(prompts[0])
        except Exception as exc:  # the table is optional evidence; never fail the bench for it
            _log(f"decode kernel table skipped: {exc!r}")
    # optional: per-kernel device time of one request's prefill (profiler;
    # not a timing of record), every rank in step
    ptable = None
    if os.environ.get("KVSERVE_PROFILE_PREFILL", "1") != "0":
        try:
            ptable = engine.prefill_kernel_table(prompts[0])
        except Exception as exc:  # optional evidence; never fail the bench for it
            _log(f"prefill kernel table skipped: {exc!r}")
    wire = None
    if ctx.is_prefill and profile.lossless:
        torch.cuda.synchronize()
        wire = int(sum(int(x.wire_bytes.item()) for x in engine.xfer_sets["default"]))
    mine = {"steps": [t.__dict__ for t in timings], "handoff": handoffs, "wire": wire, "ktable": ktable,
            "ptable": ptable if ctx.is_prefill else None}
    allr = [None] * ctx.world_size
    if ctx.distributed:
        dist.all_gather_object(allr, mine, group=ctx.cpu_group)
    else:
        allr = [mine]
    allt = [r["steps"] for r in allr]
    out = None
    if ctx.rank == 0:
        def col(step, key):
            vals = [allt[r][step][key] for r in range(len(allt))]
            vals = [v for v in vals if not (isinstance(v, float) and math.isnan(v))]
            return max(vals) if vals else float("nan")
        def col_min(step, key):
            vals = [allt[r][step][key] for r in range(len(allt))]
            vals = [v for v in vals if not (isinstance(v, float) and math.isnan(v))]
            return min(vals) if vals else float("nan")
        ttft = [col(s, "first_token") for s in range(args.steps)]
        end = [col(s, "all_done") for s in range(args.steps)]
        prefill = [col(s, "prefill_done") for s in range(args.steps)]
        ingest = [col(s, "ingest_done") for s in range(args.steps)]
        kv_exposed = [max(0.0, ingest[s] - prefill[s]) for s in range(args.steps)]
        # layer 0's encode start (earliest prefill rank) -> last layer ingested (latest decode rank)
        kv_handoff = [ingest[s] - col_min(s, "encode_start") for s in range(args.steps)]
        iso = [max(allr[r]["handoff"][i]["ingest_ms"] for r in range(len(allr))
                   if not math.isnan(allr[r]["handoff"][i]["ingest_ms"])) for i in range(len(handoffs))]
        payload = timings[0].payload_bytes if ctx.is_prefill else allt[0][0]["payload_bytes"]
        raw = allt[0][0]["raw_bytes"]
        tp = max(1, ctx.world_size // 2)
        ttft_p50 = statistics.median(ttft)
        decode_ms = [end[s] - ttft[s] for s in range(args.steps)]
        launches = sum(allt[r][s]["launches"] for r in range(len(allt)) for s in range(args.steps))
        e2e_ttft = [col(s, "first_token_host") for s in range(args.steps)]
        e2e_req = [col(s, "request_host") for s in range(args.steps)]
        out = {
            "metric": BASELINE_METRIC,
            "value": round(ttft_p50, 3),
            "unit": "ms (TTFT p50)",
            "n_gpus": args.gpus,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(statistics.mean(end), 3),
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (random-init weights of the named architecture, uniform-random prompt token ids)",
            "impl": "ours",
            "kv_transfer_ms_p50": round(statistics.median(iso), 3),
            "kv_transfer": {
                "definition": "one request's KV hand-off on its own: all layers encoded, pushed and decoded into "
                              "the paged cache, device time from a common start to the last layer ingested, max "
                              "over ranks (median of %d)" % len(iso),
                "roofline_ms": round(_handoff_roofline_ms(raw, payload, ctx.world_size), 4),
                "fraction_of_roofline": round(_handoff_roofline_ms(raw, payload, ctx.world_size)
                                              / statistics.median(iso), 3),
                "roofline": "max((raw + payload bytes) per GPU side / measured HBM copy GB/s, payload / 770 GB/s "
                            "NVLink per direction); colocated: both sides on one GPU",
            },
            "kv_transfer_exposed_ms_p50": round(statistics.median(kv_exposed), 3),
            "kv_handoff_ms_p50": round(statistics.median(kv_handoff), 3),
            "recon": recon,
            "prefill_ms_p50": round(statistics.median(prefill), 3),
            "kv_ready_ms_p50": round(statistics.median(ingest), 3),
            "decode_ms_per_token": round(statistics.median(decode_ms) / max(1, args.max_new - 1), 4),
            "kv_payload_bytes_per_request": int(payload) * tp,
            "kv_raw_bytes_per_request": int(raw) * tp,
            "compression_ratio": round(raw / payload, 3) if payload else None,
            "kv_wire_bytes_per_request": (sum(r["wire"] for r in allr if r["wire"] is not None)
                                          if any(r["wire"] is not None for r in allr) else None),
            "config": {"model": cfg.name, "layers": cfg.num_layers, "global_batch": 1,
                       "seq_len": args.prompt_len, "max_new_tokens": args.max_new,
                       "parallelism": ("colocated-1gpu" if ctx.world_size == 1 else f"{tp}P{tp}D-tp{tp}")
                                      if n_rep == 1 else
                                      f"dp{n_rep}x" + ("colocated" if ctx.world_size == 1 else f"{tp}P{tp}D-tp{tp}"),
                       "profile": args.profile, "link_gbps": args.link_gbps or None,
                       "l2": "inputs larger than L2 (%.1f GB of weights per rank, %.2f GiB raw KV per request)"
                             % (engine.model.weight_bytes() / 1e9, raw * tp / 2 ** 30)},
            "e2e": {"value": round(statistics.median(e2e_ttft), 3),
                    "unit": "ms (TTFT p50, host wall clock from PDEngine.generate() entry to the first token "
                            "on the host; prompt H2D from pinned memory and token D2H inside every step)",
                    "h2d_bytes_per_step": 4 * args.prompt_len, "d2h_bytes_per_step": 4 * (args.max_new + 1),
                    "request_ms_p50": round(statistics.median(e2e_req), 3),
                    "wall_ms_per_request": round(1e3 * wall_s / args.steps, 3)},
            "gpu_launches": int(launches),
            "clocks": clocks,
            "decode_kernel_table": next((r["ktable"][:16] for r in allr if r["ktable"]), None),
            "prefill_kernel_table": next((r["ptable"][:16] for r in allr if r["ptable"]), None),
            "_ttft": ttft, "_e2e": e2e_ttft,
        }
    if n_rep > 1:
        # every replica served its own requests: TTFT p50 over all of them,
        # launches summed, the rest from replica 0
        allo = [None] * ctx.job_world_size
        dist.all_gather_object(allo, out if ctx.rank == 0 else None, group=ctx.job_cpu_group)
        reps = [o for o in allo if o is not None]
        if ctx.global_rank == 0:
            out = dict(reps[0])
            out["value"] = round(statistics.median([t for o in reps for t in o["_ttft"]]), 3)
            out["e2e"] = dict(out["e2e"], value=round(statistics.median([t for o in reps for t in o["_e2e"]]), 3))
            out["gpu_launches"] = int(sum(o["gpu_launches"] for o in reps))
            out["replica_ttft_ms_p50"] = [o["value"] for o in reps]
            out["clocks"] = clocks
    if ctx.global_rank == 0:
        out.pop("_ttft", None)
        out.pop("_e2e", None)
        _emit(out)
    engine.close()
    destroy_parallel(ctx)


if __name__ == "__main__":
    main()
