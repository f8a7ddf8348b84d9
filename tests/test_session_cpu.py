"""Chunked compression-session protocol on CPU: message round trips, state
machine rules, token accounting, a full producer/consumer exchange over
ZeroMQ (in-process and through the helper process), abort, timeouts and
the bootstrap registry."""
import socket
import time

import pytest
import torch

from kvserve_b200.session import (ChunkPull, ChunkReady, IllegalTransition, ReceiveSlot, ReceiveSlotState,
                                  SessionOpen, SessionState, XferMetadata, chunk_token_counts, decode_request,
                                  decode_response, encode_message, suffix_token_counts)
from kvserve_b200.session.service import ConsumerService, ProducerService
from kvserve_b200.session.state import ConsumerSession


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_messages_round_trip_and_are_tagged():
    meta = XferMetadata("d0", 1234, 2, 1, {"t1": ("r1", [[3, 4, 5]])}, arena_ipc_handle=b"\x01\x02",
                        slot_bytes=4096, num_slots=2)
    for m in (SessionOpen(meta, "n1"), ChunkPull("t1", "r1", 0, 1, 4096, 1, "n1")):
        assert decode_request(encode_message(m)) == m
    r = ChunkReady(0, 100, 20)
    assert decode_response(encode_message(r)) == r


def test_state_machines_reject_illegal_transitions():
    slot = ReceiveSlot(0)
    with pytest.raises(IllegalTransition):
        slot.move(ReceiveSlotState.DECODING)
    slot.move(ReceiveSlotState.GRANTED, chunk_id=3, owner="t")
    slot.move(ReceiveSlotState.RECEIVED)
    slot.move(ReceiveSlotState.FREE)
    assert slot.chunk_id is None and slot.owner is None
    s = ConsumerSession("t", "r")
    s.move(SessionState.OPENING)
    s.move(SessionState.ACTIVE)
    s.move(SessionState.COMPLETE)
    with pytest.raises(IllegalTransition):
        s.move(SessionState.ACTIVE)


def test_token_accounting_with_prefix_hit():
    # 100 tokens = 7 blocks of 16; D already holds 4 blocks, asks for 3
    assert suffix_token_counts(100, [[7, 8, 9]], {0: 16}) == {0: 100 - 4 * 16}
    assert suffix_token_counts(100, [[]], {0: 16}) == {0: 0}
    assert chunk_token_counts({0: 36}, {0: 16}, 0, 2) == {0: 32}
    assert chunk_token_counts({0: 36}, {0: 16}, 2, 2) == {0: 4}


def _exchange(n_blocks, slots, per_chunk=1):
    """Producer 'encodes' chunk c of a source tensor into a shared arena
    slot; the consumer 'decodes' the slot into its destination."""
    ep = f"tcp://127.0.0.1:{_port()}"
    src = torch.arange(n_blocks * 16, dtype=torch.float32).view(n_blocks, 16)
    arena = torch.zeros(slots, per_chunk * 16)
    dst = torch.zeros_like(src)

    def enc(sess, pull):
        lo = pull.chunk_id * per_chunk
        rows = src[lo:lo + per_chunk].reshape(-1)
        arena[pull.slot_id, :rows.numel()] = rows
        return rows.numel() * 4, rows.numel() * 4

    def dec(sess, slot, ready):
        lo = ready.chunk_id * per_chunk
        n = ready.payload_bytes // 4
        dst[lo:lo + n // 16] = arena[slot.slot_id, :n].view(-1, 16)

    done = []
    prod = ProducerService(ep, enc)
    cons = ConsumerService("d0", slots, per_chunk * 64, dec, done.append)
    prod.add_send("t1", [list(range(n_blocks))], n_blocks * 16)
    cons.open(ep, "t1", "r1", [list(range(100, 100 + n_blocks))], n_blocks * 16,
              logical_blocks_per_chunk=per_chunk)
    deadline = time.monotonic() + 20
    while not done and time.monotonic() < deadline:
        prod.poll(2)
        cons.poll(2)
    prod.close()
    cons.close()
    return src, dst, done, cons, prod


def test_producer_consumer_exchange_reuses_slots():
    src, dst, done, cons, prod = _exchange(n_blocks=7, slots=2, per_chunk=2)
    assert done and done[0].state is SessionState.COMPLETE and done[0].total_chunks == 4
    assert torch.equal(src, dst)
    assert all(s.state is ReceiveSlotState.FREE for s in cons.slots)
    assert prod.stats["pulls"] == 4 and cons.stats["chunks"] == 4


def test_unknown_transfer_fails_session_and_abort_is_acknowledged():
    ep = f"tcp://127.0.0.1:{_port()}"
    prod = ProducerService(ep, lambda s, m: (0, 0), open_timeout_s=0.5)
    done = []
    cons = ConsumerService("d0", 1, 64, lambda *a: None, done.append)
    cons.open(ep, "missing", "r", [[1]], 16)     # never registered: refused after the open timeout
    t0 = time.monotonic()
    while not done and time.monotonic() - t0 < 10:
        prod.poll(2)
        cons.poll(2)
    assert done[0].state is SessionState.FAILED and "unknown" in done[0].error
    prod.add_send("t2", [[0, 1]], 32)
    cons.open(ep, "t2", "r2", [[5, 6]], 32)
    cons.abort("t2", "client went away")
    t0 = time.monotonic()
    while "t2" in prod.sessions and time.monotonic() - t0 < 10:
        prod.poll(2)
    assert prod.finished[-1].state is SessionState.CANCELLED
    prod.close()
    cons.close()


def test_open_before_registration_waits_for_the_send():
    ep = f"tcp://127.0.0.1:{_port()}"
    prod = ProducerService(ep, lambda s, m: (64, 8), open_timeout_s=10.0)
    done = []
    cons = ConsumerService("d0", 1, 64, lambda *a: None, done.append)
    cons.open(ep, "late", "r", [[1, 2]], 32)
    for _ in range(20):
        prod.poll(2)
        cons.poll(2)
    assert not done and "late" in prod._early
    prod.add_send("late", [[7, 8]], 32)
    t0 = time.monotonic()
    while not done and time.monotonic() - t0 < 10:
        prod.poll(2)
        cons.poll(2)
    assert done[0].state is SessionState.COMPLETE and not prod._early
    prod.close()
    cons.close()


def test_unopened_send_expires():
    ep = f"tcp://127.0.0.1:{_port()}"
    prod = ProducerService(ep, lambda s, m: (0, 0), open_timeout_s=0.0)
    prod.add_send("t", [[0]], 16)
    expired = prod.sweep(time.monotonic() + 1.0)
    assert [s.transfer_id for s in expired] == ["t"] and expired[0].state is SessionState.CANCELLED
    prod.close()


def test_helper_process_runs_jobs_in_engine_process():
    from kvserve_b200.session.process import (DecodeChunkJob, DrainSlotsJob, EncodeChunkJob, Open, AddSend,
                                              SessionProcess)
    ep = f"tcp://127.0.0.1:{_port()}"
    log = []
    prod = SessionProcess("producer", {"endpoint": ep}, {
        EncodeChunkJob: lambda j: (log.append(("enc", j.chunk_id, j.slot_id)) or (64, 16)),
        DrainSlotsJob: lambda j: None})
    cons = SessionProcess("consumer", {"name": "d0", "num_slots": 2, "slot_bytes": 64}, {
        DecodeChunkJob: lambda j: log.append(("dec", j.chunk_id, j.payload_bytes)),
        DrainSlotsJob: lambda j: None})
    try:
        prod.request(AddSend("t", [[0, 1, 2]], 48))
        time.sleep(0.2)
        cons.request(Open(ep, "t", "r", [[9, 10, 11]], 48))
        t0 = time.monotonic()
        while not cons.done and time.monotonic() - t0 < 30:
            prod.serve_jobs(0.01)
            cons.serve_jobs(0.01)
        assert cons.done and cons.done[0].state == "COMPLETE" and cons.done[0].completed_chunks == 3
        assert sorted(x[1] for x in log if x[0] == "enc") == [0, 1, 2]
        assert all(x[2] == 16 for x in log if x[0] == "dec")
    finally:
        prod.stop()
        cons.stop()


def test_bootstrap_registry_and_stats():
    from fastapi.testclient import TestClient
    from kvserve_b200.session.bootstrap import TransferStats, make_app
    client = TestClient(make_app())
    assert client.post("/register", json={"engine_id": "p0", "tp_rank": 1, "endpoint": "tcp://h:1",
                                          "tp_size": 2}).json() == {"ok": True}
    assert client.get("/query", params={"engine_id": "p0", "tp_rank": 1}).json()["endpoint"] == "tcp://h:1"
    assert client.get("/query", params={"engine_id": "nope"}).status_code == 404
    assert client.delete("/engine/p0").json() == {"removed": 1}
    st = TransferStats()
    st.record(0.5, 2 ** 20, 2)
    st.record(1.5, 3 * 2 ** 20, 4)
    st.record_failure()
    r = st.reduce()
    assert r["num_transfers"] == 2 and r["failed"] == 1 and abs(r["total_mb"] - 4) < 1e-9


def test_heterogeneous_tp_plan_covers_every_head_once():
    from kvserve_b200.session.tp_plan import (head_shard, source_ranks, target_ranks, tp_ratio, transfer_plan,
                                              validate_region_lengths)
    assert tp_ratio(4, 2) == 2 and tp_ratio(2, 4) == -2 and tp_ratio(2, 2) == 1
    import pytest
    with pytest.raises(ValueError):
        tp_ratio(3, 2)
    for H in (8, 4, 2):
        for p in (1, 2, 4, 8):
            for c in (1, 2, 4, 8):
                if (p > H and p % H) or (c > H and c % H):
                    continue
                plan = transfer_plan(p, c, H)
                for d in range(c):
                    ds = head_shard(d, c, H)
                    got = sorted(cp.dst_head + i for cp in plan if cp.dst_rank == d for i in range(cp.heads))
                    assert got == list(range(ds.count)), (H, p, c, d, plan)
                for cp in plan:   # a copy's global heads agree on both sides
                    ps, ds = head_shard(cp.src_rank, p, H), head_shard(cp.dst_rank, c, H)
                    assert ps.first + cp.src_head == ds.first + cp.dst_head
                    assert cp.src_head + cp.heads <= ps.count and cp.dst_head + cp.heads <= ds.count
    # homogeneous: one whole-shard copy per pair
    assert transfer_plan(4, 4, 8) == [type(transfer_plan(1, 1, 8)[0])(r, r, 0, 0, 2) for r in range(4)]
    # P TP2 -> D TP1: two copies into disjoint halves; P TP1 -> D TP2: two disjoint slices
    assert [(c.src_rank, c.dst_head, c.heads) for c in transfer_plan(2, 1, 8)] == [(0, 0, 4), (1, 4, 4)]
    assert [(c.dst_rank, c.src_head, c.heads) for c in transfer_plan(1, 2, 8)] == [(0, 0, 4), (1, 4, 4)]
    assert target_ranks(0, 1, 4, 8) == [0, 1, 2, 3] and source_ranks(0, 4, 1, 8) == [0, 1, 2, 3]
    assert target_ranks(3, 4, 2, 8) == [1]
    # replicated KV heads (4 heads over TP 8): replicas alternate as senders
    plan = transfer_plan(8, 4, 4)
    assert [c.src_rank for c in plan] == [0, 3, 4, 7]     # consumer d reads replica d % 2 of its head
    plan = transfer_plan(8, 8, 4)
    assert [c.src_rank for c in plan] == list(range(8))
    assert transfer_plan(2, 1, 8)[1].byte_range(4096) == (0, 4 * 4096, 4 * 4096)
    assert validate_region_lengths([4 * 4096] * 3, [8 * 4096] * 3, 2, 1, 8) is None
    assert validate_region_lengths([4 * 4096], [4 * 4096], 2, 1, 8) is not None
    assert validate_region_lengths([1], [1, 2], 1, 1, 8) is not None
