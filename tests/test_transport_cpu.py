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
