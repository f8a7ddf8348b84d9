"""Decode-step collectives fused into the projections, across 2 and 4 GPUs
(each rank a child process on its own GPU, peer memory through CUDA IPC,
NVLS off):

* ``gemv_allreduce`` equals the NCCL all-reduce of the ranks' fp32 partial
  products within bf16 rounding, and every rank holds bitwise the same
  result, for M = 1..8 and alternating launch sites;
* ``greedy`` (LM head + argmax + exchange) picks the token of the full
  gathered bf16 logits;
* both replay correctly from a CUDA graph with the epoch bump in it.
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
    from kvserve_b200.parallel.decode_allreduce import create_decode_collectives
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    cpu = dist.new_group(list(range(world)), backend="gloo", timeout=datetime.timedelta(seconds=60))
    ctx = ParallelContext(rank=rank, world_size=world, local_rank=rank, role="decode", tp_rank=rank,
                          tp_size=world, peer_rank=rank, tp_group=dist.group.WORLD, cpu_group=cpu,
                          world_group=dist.group.WORLD)
    out = {"rank": rank, "error": None, "errs": [], "same": [], "tokens_ok": []}
    dc = None
    try:
        N, K, V = 4096, 1024, 8000
        dc = create_decode_collectives(ctx, N, V, num_sites=9, device=torch.device("cuda", rank), timeout_s=5.0)
        assert dc is not None and dc.world == world
        for i, M in enumerate((1, 3, 8, 2)):
            g = torch.Generator(device="cuda").manual_seed(100 * i + rank)
            x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g)
            w = (torch.randn(N, K, device="cuda", dtype=torch.bfloat16, generator=g) * 0.05).to(torch.bfloat16)
            y = dc.gemv_allreduce(x, w, site=i % 2).clone()
            torch.cuda.synchronize()
            assert int(dc.status[0].item()) == 0
            ref = x.float() @ w.float().T
            dist.all_reduce(ref)
            out["errs"].append(((y.float() - ref).norm() / ref.norm()).item())
            gathered = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(gathered, y)
            out["same"].append(all(torch.equal(gathered[0], t) for t in gathered))
            # greedy over a vocab-parallel head of V rows per rank
            h = torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g)
            head = torch.randn(V, K, device="cuda", dtype=torch.bfloat16, generator=g)
            tok = dc.greedy(h, head, rank * V, site=8)
            logits = ops.linear(h, head)
            allv = [torch.empty_like(logits) for _ in range(world)]
            dist.all_gather(allv, logits)
            full = torch.cat(allv, dim=1).float()
            out["tokens_ok"].append(bool(torch.equal(tok.long().cpu(), full.argmax(1).cpu())))
            dc.bump()
        # a 70B-like down projection at M = 8: x takes 112 KB of shared memory,
        # one CTA fits per SM, so each CTA must take several 16-row chunks
        dc2 = create_decode_collectives(ctx, 8192, V, num_sites=2, device=torch.device("cuda", rank), timeout_s=5.0)
        g = torch.Generator(device="cuda").manual_seed(7 + rank)
        x = torch.randn(8, 7168, device="cuda", dtype=torch.bfloat16, generator=g)
        w = (torch.randn(8192, 7168, device="cuda", dtype=torch.bfloat16, generator=g) * 0.02).to(torch.bfloat16)
        y = dc2.gemv_allreduce(x, w, site=0).clone()
        torch.cuda.synchronize()
        assert int(dc2.status[0].item()) == 0
        ref = x.float() @ w.float().T
        dist.all_reduce(ref)
        out["errs"].append(((y.float() - ref).norm() / ref.norm()).item())
        gathered = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(gathered, y)
        out["same"].append(all(torch.equal(gathered[0], t) for t in gathered))
        torch.cuda.synchronize()
        dist.barrier(group=cpu)
        dc2.close()
        # graph replay: capture one step (all-reduce, greedy, bump) and replay it
        x = torch.randn(1, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
        h = torch.randn(1, K, device="cuda", dtype=torch.bfloat16)
        head = torch.randn(V, K, device="cuda", dtype=torch.bfloat16)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            dc.gemv_allreduce(x, w, site=0)
            dc.greedy(h, head, rank * V, site=8)
            dc.bump()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        dist.barrier(group=cpu)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            yg = dc.gemv_allreduce(x, w, site=0)
            tg = dc.greedy(h, head, rank * V, site=8)
            dc.bump()
        for _ in range(3):
            x.copy_(torch.randn_like(x))
            graph.replay()
            torch.cuda.synchronize()
            ref = x.float() @ w.float().T
            dist.all_reduce(ref)
            out["errs"].append(((yg.float() - ref).norm() / ref.norm()).item())
        assert int(dc.status[0].item()) == 0
        torch.cuda.synchronize()
        del graph
        dist.barrier(group=cpu)
    except Exception as exc:  # reported to the parent
        import traceback
        out["error"] = traceback.format_exc()[-2000:]
    finally:
        if dc is not None:
            torch.cuda.synchronize()
            dist.barrier(group=cpu)
            dc.close()
        dist.destroy_process_group()
    q.put(out)


@pytest.mark.parametrize("world", [2, 4])
def test_decode_collectives_match_nccl(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in ps]
    for p in ps:
        p.join(60)
    for r in res:
        assert r["error"] is None, r["error"]
        assert all(e < 1e-2 for e in r["errs"]), r["errs"]
        assert all(r["same"]) and all(r["tokens_ok"]), r
