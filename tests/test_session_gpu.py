"""The chunked session protocol on the GPU data path: a consumer process
grants slots of its CUDA-IPC receive arena, the producer process's encode
job runs the compression runtime's fused encode of each pulled chunk
straight into the granted slot (peer stores on two GPUs; IPC-mapped local
memory when there is one), and the consumer's decode job writes the chunk
into its paged blocks.  The result must be bitwise the one of the same
runtime round trip done in one process (whose kernels the runtime tests
check against the CPU oracle); an aborted session leaves every slot free."""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

L, H, D, BS, NB, PER_CHUNK, TOKENS = 3, 4, 128, 16, 48, 4, 16 * 10 + 7
SRC_BLOCKS = list(range(3, 3 + 11))
DST_BLOCKS = list(range(30, 30 + 11))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _runtime(pipeline, execution, device):
    from kvserve_b200.compression.runtime import CacheSpec, CompressionConfig, build_memory_plan, create_runtime
    cfg = CompressionConfig.from_extra_config({"compression": {
        "enable-compression-pipeline": True, "pipeline": pipeline, "logical_blocks_per_chunk": PER_CHUNK,
        "high_key_num_levels": 16, "low_key_num_levels": 16, "high_value_num_levels": 4,
        "low_value_num_levels": 4}})
    specs = {f"l{i}": CacheSpec(i, BS, H, D, torch.bfloat16) for i in range(L)}
    plan = build_memory_plan(cfg, specs, num_layers=L, device=device)
    return create_runtime(plan, "NHD", 1, device), specs


def _caches(device, fill):
    g = torch.Generator(device=device).manual_seed(9)
    mk = (lambda: torch.randn((2, NB, BS, H, D), dtype=torch.bfloat16, device=device, generator=g)) if fill else \
        (lambda: torch.zeros((2, NB, BS, H, D), dtype=torch.bfloat16, device=device))
    return {f"l{i}": mk() for i in range(L)}


def _producer(dev, port, pipeline, q):
    torch.cuda.set_device(dev)
    from kvserve_b200.session.gpu_jobs import RuntimeEncodeJob
    from kvserve_b200.session.service import ProducerService
    out = {"error": None}
    try:
        rt, _ = _runtime(pipeline, "encode", f"cuda:{dev}")
        rt.bind_kv_caches(_caches(f"cuda:{dev}", True))
        job = RuntimeEncodeJob(rt, BS, PER_CHUNK)
        prod = ProducerService(f"tcp://127.0.0.1:{port}", job)
        prod.add_send("t1", [SRC_BLOCKS], TOKENS)
        prod.add_send("t2", [SRC_BLOCKS], TOKENS)
        deadline = time.monotonic() + 120
        while (len(prod.finished) < 2) and time.monotonic() < deadline:
            prod.poll(5)
        out["finished"] = sorted((s.transfer_id, s.state.name) for s in prod.finished)
        out["stats"] = dict(prod.stats)
        job.close()
        prod.close()
    except Exception:  # noqa: BLE001
        import traceback
        out["error"] = traceback.format_exc()
    q.put(("producer", out))


def _consumer(dev, port, pipeline, q):
    torch.cuda.set_device(dev)
    from kvserve_b200.session.gpu_jobs import ReceiveArena, RuntimeDecodeJob, part_bytes
    from kvserve_b200.session.service import ConsumerService
    from kvserve_b200.session.state import ReceiveSlotState
    out = {"error": None}
    try:
        device = f"cuda:{dev}"
        rt, _ = _runtime(pipeline, "decode", device)
        dst = _caches(device, False)
        rt.bind_kv_caches(dst)
        arena = ReceiveArena(2, 2 * part_bytes(rt), device)
        done = []
        cons = ConsumerService("d0", 2, arena.slot_bytes, RuntimeDecodeJob(rt, arena, BS, PER_CHUNK), done.append,
                               arena_ipc_handle=arena.handle)
        ep = f"tcp://127.0.0.1:{port}"
        cons.open(ep, "t1", "r1", [DST_BLOCKS], TOKENS, block_size=BS, logical_blocks_per_chunk=PER_CHUNK)
        deadline = time.monotonic() + 120
        while not done and time.monotonic() < deadline:
            cons.poll(5)
        out["state"] = done[0].state.name if done else "TIMEOUT"
        # the same transfer through one process: encode into a local buffer, decode it
        ref_rt, _ = _runtime(pipeline, "both", device)
        src = _caches(device, True)
        ref_dst = _caches(device, False)
        ref_rt.bind_kv_caches(src)
        ref_rt2, _ = _runtime(pipeline, "both", device)
        ref_rt2.bind_kv_caches(ref_dst)
        for c in range(-(-len(SRC_BLOCKS) // PER_CHUNK)):
            sb, db = SRC_BLOCKS[c * PER_CHUNK:(c + 1) * PER_CHUNK], DST_BLOCKS[c * PER_CHUNK:(c + 1) * PER_CHUNK]
            valid = min(PER_CHUNK * BS, TOKENS - c * PER_CHUNK * BS)
            for part in (0, 1):
                enc = ref_rt.encode(0, {0: sb}, part, valid_tokens_by_group={0: valid})
                enc.event.synchronize()
                n = enc.codec_bytes
                ref_rt2.receive_buffer(0)[:n].copy_(enc.payload[:n])
                ref_rt2.decode(0, {0: db}, part, codec_bytes=n, valid_tokens_by_group={0: valid}).synchronize()
        idx = torch.tensor(DST_BLOCKS, device=device)
        out["equal"] = all(torch.equal(dst[n].index_select(1, idx).reshape(2, -1, H, D)[:, :TOKENS],
                                       ref_dst[n].index_select(1, idx).reshape(2, -1, H, D)[:, :TOKENS])
                           for n in dst)
        out["nonzero"] = bool(dst["l0"].abs().sum() > 0)
        # abort a second session before it completes: its slots come back free
        cons.open(ep, "t2", "r2", [DST_BLOCKS], TOKENS, block_size=BS, logical_blocks_per_chunk=PER_CHUNK)
        cons.abort("t2", "client went away")
        for _ in range(50):
            cons.poll(5)
        out["slots_free"] = all(s.state is ReceiveSlotState.FREE for s in cons.slots)
        out["chunks"] = cons.stats["chunks"]
        cons.close()
        arena.close()
    except Exception:  # noqa: BLE001
        import traceback
        out["error"] = traceback.format_exc()
    q.put(("consumer", out))


@pytest.mark.parametrize("pipeline", [["transformer", "quantizer"], ["transformer", "quantizer", "codec"]])
def test_session_moves_chunks_through_ipc_arena(pipeline):
    devs = (0, 1) if torch.cuda.device_count() > 1 else (0, 0)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_producer, args=(devs[0], port, pipeline, q)),
             ctx.Process(target=_consumer, args=(devs[1], port, pipeline, q))]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    for r in res.values():
        assert r["error"] is None, r["error"]
    c = res["consumer"]
    assert c["state"] == "COMPLETE" and c["equal"] and c["nonzero"]
    assert c["chunks"] == 3 and c["slots_free"]
    assert ("t1", "COMPLETE") in res["producer"]["finished"]
