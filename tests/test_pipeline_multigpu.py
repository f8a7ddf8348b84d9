"""Pipelined PD serving on two GPUs (1P1D): the prefill rank runs later
requests while the decode rank decodes earlier ones in one continuous batch,
with two receive slots whose device credits pace the prefill side.

* every request gets all its tokens, and its first token equals the one of
  the one-request-at-a-time path (the prefill samples it; same weights);
* the batched greedy continuation agrees with the serial one (the batched
  paged-attention split of the context can move a near-tie, so agreement is
  checked in aggregate, not bit for bit);
* with more requests than slots the credit protocol completes without a
  device timeout (the status word stays clear).
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


def _worker(rank, world, port, prompts, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from kvserve_b200.engine.pd import PDEngine
    from kvserve_b200.engine.pipeline import PipelinedServer, Request, merge_records
    from kvserve_b200.engine.transfer import TransferProfile
    from kvserve_b200.models.config import get_config
    from kvserve_b200.parallel.context import destroy_parallel, init_parallel
    out = {"rank": rank, "serial": [], "piped": None, "error": None}
    ctx = init_parallel("nccl", timeout_s=60)
    prof = TransferProfile(compressed=True, hybrid_ratio=0.0, key_levels=(16, 16), value_levels=(4, 4))
    eng = PDEngine(get_config("tiny-gqa"), ctx, prof, max_prompt=256, max_new_tokens=8, ingest_timeout_s=5.0,
                   num_slots=2, max_batch=4)
    try:
        for p in prompts:
            out["serial"].append(eng.generate(p, 8).tokens)
        server = PipelinedServer(eng, max_batch=4, timeout_s=60)
        reqs = [Request(i, p, 8, arrival_s=0.002 * i) for i, p in enumerate(prompts)]
        recs = merge_records(ctx, server.serve(reqs))
        out["piped"] = [(r.tokens, r.first_token_ms, r.done_ms) for r in recs]
    except Exception as exc:  # noqa: BLE001
        import traceback
        out["error"] = traceback.format_exc()
    q.put(out)
    torch.cuda.synchronize()
    eng.close()
    destroy_parallel(ctx)


def test_pipelined_serving_matches_serial():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 4096, (n,), generator=g, dtype=torch.int32) for n in (200, 64, 250, 17, 128, 96)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, prompts, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r["rank"]: r for r in (q.get(timeout=600) for _ in procs)}
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    for r in res.values():
        assert r["error"] is None, r["error"]
    serial, piped = res[1]["serial"], res[1]["piped"]
    assert len(piped) == len(prompts)
    agree = total = 0
    for s, (tok, ttft, done) in zip(serial, piped):
        assert tok is not None and len(tok) == 8
        assert tok[0] == s[0]
        assert ttft == ttft and done >= ttft > 0
        agree += sum(a == b for a, b in zip(tok, s))
        total += len(s)
    assert agree >= 0.9 * total, (agree, total)
