"""The credit-based PD transport over a 2-process gloo data plane (CPU).

Failures are injected on the host only: refused credits, a dropped control
reply (the producer's control timeout fires), a consumer that never starts.
"""
import multiprocessing as mp
import os
import socket
import time

import pytest
import torch


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _consumer(port, q, capacity, faults_env, expect):
    os.environ["KVSERVE_FAULTS"] = faults_env
    from kvserve_b200.transport.nccl_transport import NcclTransport
    t = NcclTransport(False, "127.0.0.1", port, data_plane="gloo", recv_buffer_size=capacity)
    got = {}
    deadline = time.time() + 60
    while len(got) < expect and time.time() < deadline:
        for rid, items in t.drain_received().items():
            for names, payload in items:
                got[rid] = (names, payload)
                t.release_received(rid, t.payload_nbytes(payload))
        time.sleep(0.01)
    out = {}
    for rid, (names, payload) in got.items():
        if payload is None:
            out[rid] = None
        elif isinstance(payload, dict):
            out[rid] = ("bundle", names, payload["meta"], [x.sum().item() for x in payload["body_chunks"]],
                        [x.sum().item() for x in payload["aux_tensors"]])
        else:
            out[rid] = ("raw", names, payload.sum().item(), list(payload.shape))
    q.put(out)
    q.close()
    q.join_thread()            # the report is out before the transport is torn down
    time.sleep(0.5)
    t.close()


def _producer(port, q, n_raw):
    from kvserve_b200.transport.nccl_transport import NcclTransport
    t = NcclTransport(True, "127.0.0.1", port, data_plane="gloo", control_timeout_s=20)
    for i in range(n_raw):
        t.send(f"r{i}", ["l0", "l1"], torch.full((4, 1000), float(i)))
    t.send_bundle("b0", ["__compressed__", "l0"], {"k": 1}, [torch.ones(10, dtype=torch.uint8)],
                  [torch.arange(4, dtype=torch.int16)])
    ok = t.wait_for_sent(timeout=60)
    q.put(ok)
    q.close()
    q.join_thread()
    time.sleep(1.0)
    t.close()


def _run(capacity=10_000_000, faults="", n_raw=3):
    ctx = mp.get_context("spawn")
    port = _free_port()
    qc, qp = ctx.Queue(), ctx.Queue()
    c = ctx.Process(target=_consumer, args=(port, qc, capacity, faults, n_raw + 1))
    p = ctx.Process(target=_producer, args=(port, qp, n_raw))
    c.start()
    time.sleep(0.5)
    p.start()
    res = qc.get(timeout=120)
    ok = qp.get(timeout=120)
    p.join(30)
    c.join(30)
    for proc in (p, c):
        if proc.is_alive():
            proc.kill()
    return res, ok


def test_raw_and_bundle_delivery():
    res, ok = _run()
    assert ok
    assert res["r2"] == ("raw", ["l0", "l1"], 8000.0, [4, 1000])
    assert res["b0"][0] == "bundle" and res["b0"][2] == {"k": 1} and res["b0"][3] == [10] and res["b0"][4] == [6]


def test_credit_retry_then_delivery():
    # tiny capacity: every payload is oversize -> admitted only into an empty buffer;
    # plus two refused credits injected on the host
    res, ok = _run(capacity=100, faults="refuse_credit:2")
    assert ok
    assert set(res) == {"r0", "r1", "r2", "b0"}


def test_zmq_transport_roundtrip_without_pickle():
    import socket
    import time
    from kvserve_b200.transport.zmq_transport import ZmqTransport
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    rx = ZmqTransport(False, "127.0.0.1", port)
    tx = ZmqTransport(True, "127.0.0.1", port)
    try:
        kv = torch.randn(3, 2, 7, 32).to(torch.bfloat16)
        tx.send("req-a", ["l0", "l1", "l2"], kv)
        tx.send("req-b", ["l0"], torch.arange(10, dtype=torch.int32))
        got = {}
        for _ in range(100):
            got.update(rx.drain_received())
            if len(got) == 2:
                break
            time.sleep(0.02)
        assert got["req-a"][0] == ["l0", "l1", "l2"] and torch.equal(got["req-a"][1], kv)
        assert torch.equal(got["req-b"][1], torch.arange(10, dtype=torch.int32))
        assert rx.drain_received() == {}
    finally:
        tx.close()
        rx.close()


def test_logger_levels(capsys):
    from kvserve_b200.utils import logger
    old = logger.get_log_level()
    try:
        logger.set_log_level(logger.LogLevel.WARNING)
        logger.log_info("quiet")
        logger.log_warning("loud")
        logger.set_log_level(logger.LogLevel.ERROR)
        logger.log_error("always")
        err = capsys.readouterr().err
        assert "loud" in err and "always" in err and "quiet" not in err
    finally:
        logger.set_log_level(old)


def test_tp_allreduce_workspace_layout():
    from kvserve_b200.parallel.tp_allreduce import workspace_layout
    lay = workspace_layout(4, 8192, 4096)
    assert lay["max_tiles"] == 64 * 16
    assert lay["stage"] == 8192 * 4096 * 2
    assert lay["flags"] - lay["stage"] == 3 * 1024 * 128 * 256 * 2
    assert lay["flag_bytes"] == 4 * 1024 * 4
    assert all(lay[k] % 256 == 0 for k in ("stage", "flags", "total"))
    one = workspace_layout(1, 300, 512)
    assert one["max_tiles"] == 3 * 2 and one["flags"] == one["stage"]   # no staging with one rank
    import pytest
    with pytest.raises(ValueError):
        workspace_layout(2, 128, 1000)
    with pytest.raises(ValueError):
        workspace_layout(9, 128, 1024)


def test_tp_allreduce_not_created_without_tp():
    import torch
    from kvserve_b200.parallel.context import ParallelContext
    from kvserve_b200.parallel.tp_allreduce import create_tp_allreduce
    assert create_tp_allreduce(ParallelContext(), 128, 1024, torch.device("cpu")) is None


def test_ipc_receive_pool_ranges():
    """First-fit ranges of the CUDA-IPC data plane's receive pool: aligned,
    disjoint, refused when full, coalesced again when freed."""
    from kvserve_b200.transport.nccl_transport import _RangePool
    p = _RangePool(4096)
    a = p.alloc(100)
    b = p.alloc(1000)
    c = p.alloc(256)
    assert (a, b, c) == (0, 256, 1280) and all(x % 256 == 0 for x in (a, b, c))
    assert p.alloc(4096) is None
    p.free(b, 1000)
    assert p.alloc(700) == 256          # first fit reuses the hole
    p.free(a, 100)
    p.free(256, 700)
    p.free(c, 256)
    assert p.free_bytes() == 4096 and p.alloc(4096) == 0


def test_pipeline_host_helpers():
    """Bucket choice, Poisson schedule and record merging of the pipelined
    server (host logic; the serving loops themselves need two GPUs)."""
    from kvserve_b200.engine.pipeline import RequestRecord, bucket_for, merge_records, poisson_schedule
    from kvserve_b200.parallel.context import ParallelContext
    assert [bucket_for(n) for n in (1, 2, 3, 4, 5, 8)] == [1, 2, 4, 4, 8, 8]
    with pytest.raises(ValueError):
        bucket_for(9)
    a = poisson_schedule(200, 4.0, seed=1)
    assert a == sorted(a) and a == poisson_schedule(200, 4.0, seed=1)
    assert 30 < a[-1] < 80            # mean gap 0.25 s
    assert poisson_schedule(3, 0.0) == [0.0, 0.0, 0.0]
    recs = [RequestRecord(0, 0.0, first_token_ms=5.0)]
    assert merge_records(ParallelContext(), recs) is recs


def test_channel_control_block_layout():
    """Per-slot control words: layer flags, first token, its flag, the
    credit, one pad word — the producer and consumer views agree."""
    from kvserve_b200.transport.p2p import ctrl_words
    assert ctrl_words(32) == 36


def test_trace_stamp_decoding():
    """Starts are stored as ~t (atomic max keeps the earliest), ends as t;
    zero means not stamped."""
    import math
    from kvserve_b200.utils.trace import decode_stamps, summarize_stamps
    mask = (1 << 64) - 1
    base = 1_700_000_000_000_000_000
    enc = lambda t: (~t) & mask  # noqa: E731
    signed = lambda u: u - (1 << 64) if u >= (1 << 63) else u  # noqa: E731
    raw = torch.tensor([[signed(enc(base)), base + 2_000_000, signed(enc(base + 1_000_000)), base + 3_000_000],
                        [signed(enc(base + 500_000)), base + 2_500_000, 0, 0]], dtype=torch.int64)
    st = decode_stamps(raw)
    assert st["base_ns"] == base
    assert st["layers_ms"][0] == [0.0, 2.0, 1.0, 3.0]
    assert st["layers_ms"][1][:2] == [0.5, 2.5] and math.isnan(st["layers_ms"][1][2])
    assert summarize_stamps(st) == {"encode_span_ms": 2.5, "ingest_span_ms": 2.0}


def _replica_worker(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import torch.distributed as dist
    from kvserve_b200.parallel.context import destroy_parallel, init_parallel
    ctx = init_parallel("gloo", timeout_s=60, replicas=2)
    # a broadcast inside the replica from its local rank 0 (global rank rank_offset)
    t = torch.tensor([float(ctx.replica * 10 + ctx.rank)])
    dist.broadcast(t, src=ctx.rank_offset, group=ctx.cpu_group)
    allr = [None] * ctx.job_world_size
    dist.all_gather_object(allr, ctx.global_rank, group=ctx.job_cpu_group)
    q.put({"rank": rank, "replica": ctx.replica, "local": ctx.rank, "world": ctx.world_size, "role": ctx.role,
           "peer": ctx.peer_rank, "offset": ctx.rank_offset, "bcast": float(t.item()), "all": allr,
           "leaders": [ctx.global_ranks("prefill"), ctx.global_ranks("decode")]})
    destroy_parallel(ctx)


def test_data_parallel_replicas_layout():
    """Four gloo ranks as two independent 1P1D replicas: replica-local ranks,
    roles and peers, replica-scoped collectives, a job-wide group."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_replica_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = {r["rank"]: r for r in (q.get(timeout=120) for _ in procs)}
    for p in procs:
        p.join(30)
    assert [res[r]["replica"] for r in range(4)] == [0, 0, 1, 1]
    assert [res[r]["role"] for r in range(4)] == ["prefill", "decode", "prefill", "decode"]
    assert [res[r]["peer"] for r in range(4)] == [1, 0, 1, 0]
    assert [res[r]["offset"] for r in range(4)] == [0, 0, 2, 2]
    assert [res[r]["bcast"] for r in range(4)] == [0.0, 0.0, 10.0, 10.0]
    assert all(res[r]["all"] == [0, 1, 2, 3] for r in range(4))
    assert res[3]["leaders"] == [[2], [3]]


def test_slot_guards_detect_an_overrun_into_the_next_slot():
    from kvserve_b200.transport.canary import GUARD_PATTERN, damaged_slots, fill_guards
    slots, payload, guard = 3, 1024, 256
    buf = torch.zeros(slots * (payload + guard), dtype=torch.uint8)
    fill_guards(buf, slots, payload + guard, payload)
    buf[:payload] = 7                              # in-bounds frames leave the guards alone
    buf[(payload + guard) + 5] = 1
    assert damaged_slots(buf, slots, payload + guard, payload) == []
    buf[2 * (payload + guard) - 3] = GUARD_PATTERN ^ 1   # slot 1 wrote 253 bytes past its end
    assert damaged_slots(buf, slots, payload + guard, payload) == [1]
    assert damaged_slots(buf, slots, payload, payload) == []   # no guards configured


def test_stats_rows_of_a_real_exchange_summarize(tmp_path):
    """Rows written by both transport ends during a gloo exchange reduce to
    per-direction counts, bytes and timing percentiles."""
    from kvserve_b200.transport.stats_summary import read_rows, summarize
    path = tmp_path / "stats.jsonl"
    os.environ["KVSERVE_TRANSPORT_STATS_PATH"] = str(path)
    try:
        res, ok = _run()
    finally:
        os.environ.pop("KVSERVE_TRANSPORT_STATS_PATH", None)
    assert ok
    with open(path, "a") as f:
        f.write('{"direction": "send", "trunc')                 # a row cut by a crashed writer is skipped
    s = summarize(read_rows([str(path)]))
    d = s["directions"]
    assert d["send"]["count"] == 4 and d["recv"]["count"] == 4
    assert d["send"]["payload_bytes"] == d["recv"]["payload_bytes"] > 0
    assert d["send"]["total_s"]["p50_ms"] <= d["send"]["total_s"]["p95_ms"] <= d["send"]["total_s"]["max_ms"]
    assert "recv_credit" in d and s["credit_retries"] >= 0


def test_llm_facade_resolves_profiles_and_is_exported():
    """The package root's ``LLM`` entry resolves transfer profiles by name,
    by connector-style profile dict or JSON file, or passes one through."""
    import kvserve_b200
    from kvserve_b200.engine.api import LLM, resolve_profile
    from kvserve_b200.engine.transfer import TransferProfile
    assert kvserve_b200.LLM is LLM
    assert resolve_profile("raw").compressed is False and resolve_profile(None).compressed is False
    k4v2 = resolve_profile("k4v2")
    assert k4v2.compressed and tuple(k4v2.value_levels) == (4, 4)
    from_file = resolve_profile("configs/compression/hadamard_k4v2_bitpack.json")
    assert from_file.compressed
    p = TransferProfile.raw()
    assert resolve_profile(p) is p
    with pytest.raises(ValueError):
        resolve_profile(3.14)
