"""Row-parallel projection + all-reduce: fused peer-memory kernel vs GEMM + NCCL.

    python -m torch.distributed.run --nnodes 1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P -m kvserve_b200.parallel.bench_tp [--tokens 8192] [--iters 20]

For Llama-3.1-8B's attention-output (K = 4096/N) and MLP-down (K = 14336/N)
projections of a prefill chunk, rank 0 prints one JSON object: per shape the
CUDA-event ms per call (max over ranks) of ``gemm`` followed by
``torch.distributed.all_reduce`` and of the fused launch, and the roofline
time max(FLOPs / measured bf16 peak, NVLink bytes / 770 GB/s) where the
NVLink bytes per rank are 2 (N-1)/N of the output.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from .. import ops
from ..ops.microbench import peaks
from .context import init_parallel
from .tp_allreduce import create_tp_allreduce

NVLINK_GBS = 770.0   # measured peer copy per direction on this platform


def _time(fn, iters: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args(argv)
    ctx = init_parallel("nccl", timeout_s=120)
    w = ctx.world_size
    # one TP group over all ranks
    from .context import ParallelContext
    tp = ParallelContext(rank=ctx.rank, world_size=w, local_rank=ctx.local_rank, role="prefill", tp_rank=ctx.rank,
                         tp_size=w, peer_rank=ctx.rank, tp_group=dist.group.WORLD, cpu_group=ctx.cpu_group,
                         world_group=dist.group.WORLD)
    dev = torch.device("cuda", torch.cuda.current_device())
    ws = create_tp_allreduce(tp, a.tokens, a.hidden, dev)
    pk = peaks()
    M, N = a.tokens, a.hidden
    res = {"world": w, "tokens": M, "hidden": N, "peaks": pk}
    # comm_only: K = 64, the GEMM is negligible and the fused time is the
    # reduction's NVLink time
    for name, K in (("comm_only", 64), ("o_proj", 4096 // w), ("down_proj", 14336 // w)):
        A = [torch.randn(M, K, device=dev, dtype=torch.bfloat16) for _ in range(2)]
        B = [torch.randn(N, K, device=dev, dtype=torch.bfloat16) / K ** 0.5 for _ in range(2)]
        C = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        it = [0]

        def unfused():
            i = it[0] = it[0] ^ 1
            ops.gemm(A[i], B[i], C)
            dist.all_reduce(C)

        def fused():
            i = it[0] = it[0] ^ 1
            ws.gemm_allreduce(A[i], B[i])

        def gemm_only():
            i = it[0] = it[0] ^ 1
            ops.gemm(A[i], B[i], C)

        flops = 2.0 * M * N * K
        link = 2.0 * (w - 1) / w * M * N * 2
        roof = max(flops / (pk["bf16_tflops"] * 1e9), link / (NVLINK_GBS * 1e6))
        r = {"K": K, "gemm_ms": round(_time(gemm_only, a.iters), 4),
             "gemm_nccl_ms": round(_time(unfused, a.iters), 4)}
        if ws is not None:
            r["fused_ms"] = round(_time(fused, a.iters), 4)
            r["fused_frac_of_roofline"] = round(roof / r["fused_ms"], 3)
        r["roofline_ms"] = round(roof, 4)
        ops.check_device_status()
        res[name] = r
    if ctx.rank == 0:
        print(json.dumps(res))
    torch.cuda.synchronize()
    dist.barrier()
    if ws is not None:
        ws.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
