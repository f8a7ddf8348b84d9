"""Fused GEMM + tensor-parallel all-reduce across 2 and 4 GPUs (each rank a
child process on its own GPU, peer memory through CUDA IPC, NVLS off).

* every rank receives the same bf16 result, equal to the sum of the ranks'
  fp32 partial products within bf16 rounding;
* successive launches of different M reuse staging and flags (epochs);
* a TP prefill through the engine gives the tokens of the NCCL path.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    from kvserve_b200 import ops
    from kvserve_b200.parallel.context import ParallelContext
    from kvserve_b200.parallel.tp_allreduce import create_tp_allreduce
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    cpu = dist.new_group(list(range(world)), backend="gloo", timeout=datetime.timedelta(seconds=60))
    # one TP group of `world` ranks (no PD split): role "prefill" on all ranks
    ctx = ParallelContext(rank=rank, world_size=world, local_rank=rank, role="prefill", tp_rank=rank,
                          tp_size=world, peer_rank=rank, tp_group=dist.group.WORLD, cpu_group=cpu,
                          world_group=dist.group.WORLD)
    out = {"rank": rank, "error": None, "errs": [], "results": []}
    ws = None
    try:
        N, K = 4096, 1024
        ws = create_tp_allreduce(ctx, 4096, N, torch.device("cuda", rank), timeout_s=5.0)
        assert ws is not None
        for i, M in enumerate((4096, 300, 1000, 4096)):
            g = torch.Generator(device="cuda").manual_seed(100 * i + rank)
            a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g)
            b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16, generator=g)
            c = ws.gemm_allreduce(a, b).clone()
            ops.check_device_status()
            part = a.float() @ b.float().T
            ref = part.clone()
            dist.all_reduce(ref)
            out["errs"].append(((c.float() - ref).norm() / ref.norm()).item())
            out["results"].append(c.float().sum().item())
            # every rank holds the identical tensor
            other = c.clone()
            dist.broadcast(other, 0)
            out.setdefault("same", []).append(bool(torch.equal(other, c)))
        # a TP-2 prefill: fused reductions vs GEMM + NCCL all-reduce
        from kvserve_b200.models.config import get_config
        from kvserve_b200.models.llama import LlamaShard
        cfg = get_config("tiny-gqa")
        m = LlamaShard(cfg, rank, world, torch.device("cuda", rank), 0, dist.group.WORLD, max_position=1024)
        T = 300
        ids = torch.randint(0, cfg.vocab, (T,), device="cuda", dtype=torch.int32,
                            generator=torch.Generator(device="cuda").manual_seed(5))
        pos = torch.arange(T, device="cuda", dtype=torch.int32)
        kv = []
        for fused in (True, False):
            m.tp_ar = ws if fused else None
            k = torch.zeros((cfg.num_layers, T, m.hkv, m.D), device="cuda", dtype=torch.bfloat16)
            v = torch.zeros_like(k)
            tok = m.prefill(ids, pos, k, v, sample=True)
            kv.append((k, v, int(tok)))
        ops.check_device_status()
        out["prefill_err"] = max(((a.float() - b.float()).norm() / b.float().norm()).item()
                                 for a, b in ((kv[0][0][-1], kv[1][0][-1]), (kv[0][1][-1], kv[1][1][-1])))
        out["tokens"] = (kv[0][2], kv[1][2])
    except Exception as exc:  # reported to the parent
        out["error"] = f"{type(exc).__name__}: {exc}"
    torch.cuda.synchronize()
    dist.barrier(group=cpu)
    if ws is not None:
        ws.close()
    q.put(out)
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gemm_allreduce_ranks(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {r["rank"]: r for r in (q.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    for r in range(world):
        assert res[r]["error"] is None, res[r]["error"]
        assert all(e < 1e-2 for e in res[r]["errs"]), res[r]["errs"]
        assert all(res[r]["same"])
        assert res[r]["results"] == res[0]["results"]
        assert res[r]["prefill_err"] < 2e-2, res[r]["prefill_err"]
        assert res[r]["tokens"] == res[0]["tokens"]
