"""The chunked session protocol end to end on CPUs with real compressed
frames: a producer process pulls chunks of its paged cache through the CPU
runtime (Hadamard + 4-bit min-max, with and without the lossless codec)
into the consumer process's shared-memory receive arena — or, for a
consumer that exports no arena (another node), inline in the replies — and
the consumer decodes them into its blocks.  The result must equal the same
runtime round trip done in one process, bit for bit."""
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

L, H, D, BS, NB, PER_CHUNK, TOKENS = 2, 4, 128, 16, 32, 3, 16 * 8 + 5
SRC = list(range(2, 11))
DST = list(range(20, 29))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _runtime(pipeline, execution):
    from kvserve_b200.compression.runtime import CacheSpec, CompressionConfig, build_memory_plan, create_runtime
    cfg = CompressionConfig.from_extra_config({"compression": {
        "enable-compression-pipeline": True, "pipeline": pipeline, "logical_blocks_per_chunk": PER_CHUNK,
        "high_key_num_levels": 16, "low_key_num_levels": 16, "high_value_num_levels": 16,
        "low_value_num_levels": 16}})
    specs = {f"l{i}": CacheSpec(i, BS, H, D, torch.bfloat16) for i in range(L)}
    return create_runtime(build_memory_plan(cfg, specs, num_layers=L, device="cpu"), "NHD", 1, "cpu", execution=execution)


def _caches(fill):
    g = torch.Generator().manual_seed(21)
    mk = (lambda: torch.randn((2, NB, BS, H, D), generator=g)) if fill else (lambda: torch.zeros((2, NB, BS, H, D)))
    return {f"l{i}": mk().to(torch.bfloat16) for i in range(L)}


def _producer(port, pipeline, q):
    from kvserve_b200.session.cpu_jobs import CpuEncodeJob
    from kvserve_b200.session.service import ProducerService
    out = {"error": None}
    try:
        rt = _runtime(pipeline, "encode")
        rt.bind_kv_caches(_caches(True))
        job = CpuEncodeJob(rt, BS, PER_CHUNK)
        prod = ProducerService(f"tcp://127.0.0.1:{port}", job)
        prod.add_send("t1", [SRC], TOKENS)
        deadline = time.monotonic() + 120
        while not prod.finished and time.monotonic() < deadline:
            prod.poll(5)
        out["finished"] = [(s.transfer_id, s.state.name) for s in prod.finished]
        job.close()
        prod.close()
    except Exception:  # noqa: BLE001
        import traceback
        out["error"] = traceback.format_exc()
    q.put(("producer", out))


def _consumer(port, pipeline, q, inline=False):
    from kvserve_b200.session.cpu_jobs import CpuDecodeJob, SharedArena
    from kvserve_b200.session.gpu_jobs import part_bytes
    from kvserve_b200.session.service import ConsumerService
    out = {"error": None}
    arena = None
    try:
        rt = _runtime(pipeline, "decode")
        dst = _caches(False)
        rt.bind_kv_caches(dst)
        done = []
        if inline:
            slot = (2 * part_bytes(rt) + 255) // 256 * 256
            cons = ConsumerService("d0", 2, slot, CpuDecodeJob(rt, None, BS, PER_CHUNK), done.append)
        else:
            arena = SharedArena(2, 2 * part_bytes(rt))
            cons = ConsumerService("d0", 2, arena.slot_bytes, CpuDecodeJob(rt, arena, BS, PER_CHUNK), done.append,
                                   arena_ipc_handle=arena.handle)
        cons.open(f"tcp://127.0.0.1:{port}", "t1", "r1", [DST], TOKENS, block_size=BS,
                  logical_blocks_per_chunk=PER_CHUNK)
        deadline = time.monotonic() + 120
        while not done and time.monotonic() < deadline:
            cons.poll(5)
        out["state"] = done[0].state.name if done else "TIMEOUT"
        out["chunks"] = cons.stats["chunks"]
        # the same transfer in one process
        a, b = _runtime(pipeline, "both"), _runtime(pipeline, "both")
        ref_dst = _caches(False)
        a.bind_kv_caches(_caches(True))
        b.bind_kv_caches(ref_dst)
        for c in range(-(-len(SRC) // PER_CHUNK)):
            sb, db = SRC[c * PER_CHUNK:(c + 1) * PER_CHUNK], DST[c * PER_CHUNK:(c + 1) * PER_CHUNK]
            valid = min(PER_CHUNK * BS, TOKENS - c * PER_CHUNK * BS)
            for part in (0, 1):
                r = a.encode(0, {0: sb}, part, valid_tokens_by_group={0: valid})
                n = r.codec_bytes
                b.receive_buffer(0)[:n].copy_(r.payload[:n])
                b.decode(0, {0: db}, part, codec_bytes=n, valid_tokens_by_group={0: valid})
        out["equal"] = all(torch.equal(dst[n], ref_dst[n]) for n in dst)
        src = _caches(True)
        idx = torch.tensor(DST)
        got = torch.stack([dst[n].index_select(1, idx) for n in dst]).float().reshape(L, 2, -1, H, D)[:, :, :TOKENS]
        want = torch.stack([src[n].index_select(1, torch.tensor(SRC)) for n in src]).float() \
            .reshape(L, 2, -1, H, D)[:, :, :TOKENS]
        out["rel_err"] = float((got - want).norm() / want.norm())
        cons.close()
    except Exception:  # noqa: BLE001
        import traceback
        out["error"] = traceback.format_exc()
    finally:
        if arena is not None:
            arena.close()
    q.put(("consumer", out))


@pytest.mark.parametrize("inline", [False, True], ids=["shared-arena", "inline"])
@pytest.mark.parametrize("pipeline", [["transformer", "quantizer"], ["transformer", "quantizer", "codec"]])
def test_session_moves_compressed_chunks_between_cpu_processes(pipeline, inline):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_consumer, args=(port, pipeline, q, inline)),
             ctx.Process(target=_producer, args=(port, pipeline, q))]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(30)
        if p.is_alive():
            p.kill()
    for r in res.values():
        assert r["error"] is None, r["error"]
    c = res["consumer"]
    assert c["state"] == "COMPLETE" and c["chunks"] == 3 and c["equal"]
    assert c["rel_err"] < 0.15
    assert ("t1", "COMPLETE") in res["producer"]["finished"]
