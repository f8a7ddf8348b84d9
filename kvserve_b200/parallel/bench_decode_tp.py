"""Decode-step projections + collectives: fused peer-memory kernels vs GEMV + NCCL.

    python -m torch.distributed.run --nnodes 1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P -m kvserve_b200.parallel.bench_decode_tp [--model llama-3.1-8b] [--calls 64]

For one decode token (M = 1) of the model's attention-output (K = hidden/N),
MLP-down (K = intermediate/N) and LM-head (vocabulary/N rows) projections,
rank 0 prints one JSON object: per shape the device time per call (CUDA
events around a CUDA graph of ``--calls`` back-to-back calls, as a decode
step replays them; max over ranks) of

* ``gemv``: the projection alone (its weight bytes / time = streamed GB/s);
* ``gemv_nccl``: the projection followed by ``torch.distributed.all_reduce``
  (LM head: the unfused argmax + ``all_gather_into_tensor``);
* ``fused``: the single-launch kernel of ``parallel.decode_allreduce``.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from .. import ops
from ..models.config import get_config
from .context import ParallelContext, init_parallel
from .decode_allreduce import create_decode_collectives


def _graph_time_us(fn, calls: int, reps: int = 20, tail=None) -> float:
    """Per-call device time of ``calls`` back-to-back ``fn()`` in one CUDA
    graph (``tail()`` once at the end of it, e.g. the decode epoch bump)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
        if tail is not None:
            tail()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(calls):
            fn()
        if tail is not None:
            tail()
    torch.cuda.synchronize()
    dist.barrier()
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) * 1e3 / (reps * calls)], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    return float(t.item())


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--calls", type=int, default=64)
    a = ap.parse_args(argv)
    ctx = init_parallel("nccl", timeout_s=120)
    w = ctx.world_size
    tp = ParallelContext(rank=ctx.rank, world_size=w, local_rank=ctx.local_rank, role="decode", tp_rank=ctx.rank,
                         tp_size=w, peer_rank=ctx.rank, tp_group=dist.group.WORLD, cpu_group=ctx.cpu_group,
                         world_group=dist.group.WORLD)
    cfg = get_config(a.model)
    dev = torch.device("cuda", torch.cuda.current_device())
    V = cfg.vocab // w
    dc = create_decode_collectives(tp, cfg.hidden, V, num_sites=a.calls + 1, device=dev)
    res = {"world": w, "model": cfg.name, "calls_per_graph": a.calls}
    x_o = torch.randn(1, cfg.hidden // w, device=dev, dtype=torch.bfloat16)
    x_d = torch.randn(1, cfg.intermediate // w, device=dev, dtype=torch.bfloat16)
    for name, x, N in (("o_proj", x_o, cfg.hidden), ("down_proj", x_d, cfg.hidden)):
        wbytes = N * x.shape[1] * 2
        # rotate over enough weight copies that a graph's calls stream from HBM
        # (more than the 126 MB L2), as a decode step's distinct layers do
        copies = max(1, min(a.calls, -(-(256 << 20) // wbytes)))
        Ws = [torch.randn(N, x.shape[1], device=dev, dtype=torch.bfloat16) / x.shape[1] ** 0.5
              for _ in range(copies)]
        y = torch.empty(1, N, device=dev, dtype=torch.bfloat16)
        site = [0]
        nxt = [0]

        def weight():
            nxt[0] = (nxt[0] + 1) % copies
            return Ws[nxt[0]]

        def gemv():
            ops.gemv(x, weight(), y)

        def unfused():
            ops.gemv(x, weight(), y)
            dist.all_reduce(y)

        def fused():
            site[0] = (site[0] + 1) % a.calls
            dc.gemv_allreduce(x, weight(), site[0])

        r = {"K": x.shape[1], "weight_MB": round(wbytes / 1e6, 2), "weight_copies": copies,
             "gemv_us": round(_graph_time_us(gemv, a.calls), 2)}
        r["gemv_GBps"] = round(wbytes / (r["gemv_us"] * 1e3), 1)
        if w > 1:
            r["gemv_nccl_us"] = round(_graph_time_us(unfused, a.calls), 2)
            if dc is not None and dc.world > 1:
                r["fused_us"] = round(_graph_time_us(fused, a.calls, tail=dc.bump), 2)
        res[name] = r
    H = torch.randn(V, cfg.hidden, device=dev, dtype=torch.bfloat16) * 0.02
    h = torch.randn(1, cfg.hidden, device=dev, dtype=torch.bfloat16)
    vals = torch.empty(1, dtype=torch.float32, device=dev)
    both = torch.empty(2, 1, dtype=torch.float32, device=dev)
    gath = torch.empty(w, 2, 1, dtype=torch.float32, device=dev)

    def head_unfused():
        logits = ops.linear(h, H)
        idx = ops.argmax(logits, index_offset=ctx.rank * V, out_val=vals)
        if w > 1:
            both[0].copy_(vals)
            both[1].copy_(idx.float())
            dist.all_gather_into_tensor(gath, both)

    def head_fused():
        dc.greedy(h, H, ctx.rank * V, a.calls)
        dc.bump()

    r = {"rows": V, "weight_MB": round(H.numel() * 2 / 1e6, 2), "unfused_us": round(_graph_time_us(head_unfused, 8), 2)}
    if dc is not None:
        r["fused_us"] = round(_graph_time_us(head_fused, 8), 2)
    res["lm_head_greedy"] = r
    if dc is not None:
        torch.cuda.synchronize()
        assert int(dc.status[0].item()) == 0, "decode collective reported a peer timeout"
    if ctx.rank == 0:
        print(json.dumps(res))
    torch.cuda.synchronize()
    dist.barrier()
    if dc is not None:
        dc.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
