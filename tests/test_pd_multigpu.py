"""Disaggregated prefill -> decode across two GPUs (1P1D over NVLink peer
stores).  Each rank is a child process on its own GPU; NVLS is off in NCCL.

* the decode rank's greedy tokens equal those of a colocated run of the same
  weights and profile;
* a prefill rank that leaves between requests (never publishes the next
  request's frames) makes the decode rank's bounded device wait time out with
  an error status instead of hanging the GPU.
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


def _profile():
    from kvserve_b200.engine.transfer import TransferProfile
    return TransferProfile(compressed=True, hybrid_ratio=0.5, key_levels=(16, 8), value_levels=(8, 4))


def _worker(rank, world, port, prompts, mode, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from kvserve_b200.engine.pd import PDEngine
    from kvserve_b200.models.config import get_config
    from kvserve_b200.parallel.context import init_parallel, destroy_parallel
    ctx = init_parallel("nccl", timeout_s=60)
    eng = PDEngine(get_config("tiny-gqa"), ctx, _profile(), max_prompt=255, max_new_tokens=8,
                   ingest_timeout_s=2.0)
    out = {"rank": rank, "tokens": [], "error": None}
    try:
        for i, p in enumerate(prompts):
            if mode == "prefill_leaves" and i == len(prompts) - 1:
                if ctx.role == "prefill":
                    break  # leaves between requests, nothing in flight
                res = eng.generate(p, 8, sync=False)
            else:
                res = eng.generate(p, 8)
            out["tokens"].append(res.tokens)
    except RuntimeError as exc:
        out["error"] = str(exc)
    q.put(out)
    torch.cuda.synchronize()
    eng.close()
    if mode != "prefill_leaves":
        destroy_parallel(ctx)


def _run(mode, prompts):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, prompts, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    return {r["rank"]: r for r in res}


def _prompts(n):
    g = torch.Generator().manual_seed(7)
    return [torch.randint(0, 4096, (200,), generator=g, dtype=torch.int32) for _ in range(n)]


def test_1p1d_matches_colocated():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    prompts = _prompts(2)
    res = _run("normal", prompts)
    assert res[0]["error"] is None and res[1]["error"] is None
    from kvserve_b200.engine.pd import PDEngine
    from kvserve_b200.models.config import get_config
    from kvserve_b200.parallel.context import ParallelContext
    torch.cuda.set_device(0)
    col = PDEngine(get_config("tiny-gqa"), ParallelContext(), _profile(), max_prompt=255, max_new_tokens=8)
    expect = [col.generate(p, 8).tokens for p in prompts]
    col.close()
    assert res[1]["tokens"] == expect


def test_prefill_rank_leaving_is_detected_on_device():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run("prefill_leaves", _prompts(2))
    assert res[1]["error"] is not None and "timeout" in res[1]["error"]
    assert len(res[1]["tokens"]) == 1  # the first request completed normally
