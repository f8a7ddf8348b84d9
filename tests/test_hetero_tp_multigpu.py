"""Heterogeneous tensor parallelism across the KV hand-off: a TP2 prefill
group (GPUs 0-1) feeds a TP1 decode rank (GPU 2).  Each prefill rank encodes
its two KV heads into its own receive channel of the decode rank, which
decodes both frames into head offsets 0 and 2 of its paged cache.

With the raw profile the decode rank's cache must hold exactly the K/V that
the two prefill ranks computed, and the request must produce its tokens.
Needs three GPUs (NVLS off in NCCL)."""
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


def _worker(rank, world, port, prompt, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from kvserve_b200.engine.pd import PDEngine
    from kvserve_b200.engine.transfer import TransferProfile
    from kvserve_b200.models.config import get_config
    from kvserve_b200.parallel.context import destroy_parallel, init_parallel
    out = {"rank": rank, "error": None}
    ctx = init_parallel("nccl", timeout_s=60, prefill=2)
    eng = PDEngine(get_config("tiny-gqa"), ctx, TransferProfile.raw(), max_prompt=255, max_new_tokens=4,
                   ingest_timeout_s=5.0)
    try:
        T = int(prompt.numel())
        res = eng.generate(prompt, 4)
        mine = None
        if ctx.is_prefill:
            mine = (eng.k_buf[:, :T].cpu(), eng.v_buf[:, :T].cpu())
        allk = [None] * ctx.world_size
        dist.all_gather_object(allk, mine, group=ctx.cpu_group)
        if ctx.is_decode:
            out["tokens"] = res.tokens
            out["copies"] = [(c.src_rank, c.dst_head, c.heads) for c in eng.copies]
            blocks = eng.kv.allocate(T)   # the request's blocks come back first (LIFO free list)
            idx = torch.tensor(blocks, device="cuda").long()
            got = eng.kv.cache[:, :, idx].reshape(eng.cfg.num_layers, 2, -1, eng.model.hkv, eng.model.D)[:, :, :T]
            got = got.cpu()
            want_k = torch.cat([allk[0][0], allk[1][0]], dim=2)
            want_v = torch.cat([allk[0][1], allk[1][1]], dim=2)
            out["k_equal"] = bool(torch.equal(got[:, 0], want_k))
            out["v_equal"] = bool(torch.equal(got[:, 1], want_v))
            eng.kv.release(blocks)
    except Exception:  # noqa: BLE001
        import traceback
        out["error"] = traceback.format_exc()
    q.put(out)
    torch.cuda.synchronize()
    eng.close()
    destroy_parallel(ctx)


def test_tp2_prefill_to_tp1_decode_moves_head_ranges():
    if torch.cuda.device_count() < 3:
        pytest.skip("needs 3 GPUs")
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, 4096, (200,), generator=g, dtype=torch.int32)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 3, port, prompt, q)) for r in range(3)]
    for p in procs:
        p.start()
    res = {r["rank"]: r for r in (q.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    for r in res.values():
        assert r["error"] is None, r["error"]
    d = res[2]
    assert d["copies"] == [(0, 0, 2), (1, 2, 2)]
    assert d["k_equal"] and d["v_equal"]
    assert len(d["tokens"]) == 4
