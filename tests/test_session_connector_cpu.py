"""The session-protocol vLLM connector on CPU: scheduler and worker halves
of a prefill and a decode connector driven the way vLLM's scheduler and
model runner call them, with the session services on their threads over
ZeroMQ and fake encode/decode jobs that move CPU tensor blocks through a
shared arena (the GPU jobs are covered by the session GPU test).

Checked: the prefill side keeps its blocks and hands out the router's
parameters; the decode side claims an asynchronous load of the prompt,
pulls every chunk into the request's blocks and reports the request in
``get_finished``; the prefill side then reports the send; a decode engine
with a cached prefix pulls only the suffix; an unknown transfer reports its
blocks as load errors."""
import socket
import time
from types import SimpleNamespace as NS

import pytest
import torch

from kvserve_b200.connector.session_kv_connector import (KVConnectorRole, SessionConnectorMetadata,
                                                         SessionKVConnector, kv_pair, layer_index)

BS, NB, PER_CHUNK = 16, 40, 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _vllm_config(producer: bool, port: int, helper: bool = False):
    comp = {"enable-compression-pipeline": True, "pipeline": ["transformer", "quantizer"],
            "logical_blocks_per_chunk": PER_CHUNK}
    return NS(kv_transfer_config=NS(is_kv_producer=producer, kv_ip="127.0.0.1",
                                    kv_connector_extra_config={"session_port": port, "num_slots": 2,
                                                               "compression": comp, "open_timeout_s": 5.0,
                                                               "session_timeout_s": 10.0,
                                                               "session_process": helper}),
              cache_config=NS(block_size=BS), parallel_config=NS(tensor_parallel_size=1),
              model_config=NS(use_mla=False))


class FakeJobs(SessionKVConnector):
    """Encode = copy the chunk's source blocks into the granted arena slot;
    decode = copy the slot into the request's destination blocks."""
    arena: dict = {}
    seen: list = []

    def make_encode_job(self, caches):
        cache = next(iter(caches.values()))
        self._per_chunk = PER_CHUNK

        def enc(session, pull):
            ids = session.local_block_ids[0][pull.chunk_id * PER_CHUNK:(pull.chunk_id + 1) * PER_CHUNK]
            FakeJobs.seen.append((tuple(ids), session.valid_tokens_by_group[0]))
            FakeJobs.arena[pull.slot_id] = cache[:, ids].clone()
            n = FakeJobs.arena[pull.slot_id].numel() * 2
            return n, n
        return enc

    def make_decode_job(self, caches):
        cache = next(iter(caches.values()))
        self._per_chunk = PER_CHUNK

        def dec(session, slot, ready):
            ids = session.block_ids[0][ready.chunk_id * PER_CHUNK:(ready.chunk_id + 1) * PER_CHUNK]
            cache[:, ids] = FakeJobs.arena[slot.slot_id]
        return dec, 1 << 20, b""


class Blocks:
    def __init__(self, ids, unhashed):
        self.ids, self.unhashed = ids, unhashed

    def get_block_ids(self):
        return (self.ids,)

    def get_unhashed_block_ids_all_groups(self):
        return [self.unhashed]


def _req(rid, prompt_len, params, status="FINISHED_LENGTH_CAPPED"):
    return NS(request_id=rid, prompt_token_ids=list(range(prompt_len)), kv_transfer_params=params,
              status=NS(name=status))


def _pair(port, helper=False):
    src = torch.randn(2, NB, BS, 2, 64).to(torch.bfloat16)
    dst = torch.zeros_like(src)
    p_sched = FakeJobs(_vllm_config(True, port), KVConnectorRole.SCHEDULER)
    d_sched = FakeJobs(_vllm_config(False, port), KVConnectorRole.SCHEDULER)
    p_work = FakeJobs(_vllm_config(True, port, helper), KVConnectorRole.WORKER)
    d_work = FakeJobs(_vllm_config(False, port, helper), KVConnectorRole.WORKER)
    p_work.register_kv_caches({"model.layers.0.self_attn.attn": src})
    d_work.register_kv_caches({"model.layers.0.self_attn.attn": dst})
    return src, dst, p_sched, d_sched, p_work, d_work


def _sched_out(new=(), finished=()):
    """A scheduler output with ``new`` = [(req_id, block_ids, prompt_len)]
    scheduled in full this step."""
    return NS(scheduled_new_reqs=[NS(req_id=r, block_ids=(b,), num_computed_tokens=0) for r, b, _ in new],
              num_scheduled_tokens={r: n for r, _, n in new},
              scheduled_cached_reqs=NS(req_ids=[], new_block_ids=[], num_computed_tokens=[], resumed_req_ids=set()),
              finished_req_ids=set(finished))


def _step(sched, work, finished=(), so=None):
    work.bind_connector_metadata(sched.build_connector_meta(so if so is not None else _sched_out()))
    work.start_load_kv(None)
    work.wait_for_save()
    out = work.get_finished(set(finished))
    work.clear_connector_metadata()
    return out


def _prefill(p_sched, p_work, rid, tid, prompt, blocks):
    """The prefill engine: allocation, the full-prompt step, the finish."""
    req = _req(rid, prompt, {"do_remote_decode": True, "transfer_id": tid})
    p_sched.update_state_after_alloc(req, Blocks(blocks, blocks), 0)
    _step(p_sched, p_work, so=_sched_out([(rid, blocks, prompt)]))
    delay, params = p_sched.request_finished(req, blocks)
    _step(p_sched, p_work, finished={rid})
    return delay, params


def _wait_recv(d_sched, d_work, rid, timeout=20.0):
    deadline = time.monotonic() + timeout
    while time.monotonic() < deadline:
        _, recving = _step(d_sched, d_work)
        if recving and rid in recving:
            return True
        time.sleep(0.01)
    return False


def test_helpers_parse_vllm_names_and_layouts():
    assert layer_index("model.layers.17.self_attn.attn", 0) == 17
    assert layer_index("attn", 5) == 5
    t = torch.zeros(2, 3, 16, 2, 8)
    assert kv_pair(t)[0].shape == (3, 16, 2, 8)
    t2 = torch.zeros(3, 2, 16, 2, 8)
    k, v = kv_pair(t2)
    assert k.shape == (3, 16, 2, 8) and k.stride() == v.stride()


@pytest.mark.parametrize("helper", [False, True], ids=["service-thread", "helper-process"])
def test_pull_moves_every_chunk_and_both_sides_report(helper):
    """Also with the session services in helper processes (the GPU jobs
    still run in the engine processes, fed over pipes)."""
    FakeJobs.seen.clear()
    src, dst, p_sched, d_sched, p_work, d_work = _pair(_port(), helper)
    try:
        from kvserve_b200.connector.session_kv_connector import _HelperProxy
        assert isinstance(p_work._thread.service, _HelperProxy) == helper
        assert isinstance(d_work._thread.service, _HelperProxy) == helper
        prompt, p_blocks, d_blocks = 100, list(range(0, 7)), list(range(20, 27))
        delay, params = _prefill(p_sched, p_work, "p1", "t1", prompt, p_blocks)
        assert delay and params["do_remote_prefill"] and params["transfer_id"] == "t1"
        dreq = _req("d1", prompt, dict(params), status="WAITING_FOR_REMOTE_KVS")
        assert d_sched.get_num_new_matched_tokens(dreq, 0) == (prompt, True)
        d_sched.update_state_after_alloc(dreq, Blocks(d_blocks, d_blocks), prompt)
        assert dreq.kv_transfer_params["do_remote_prefill"] is False
        assert _wait_recv(d_sched, d_work, "d1")
        assert torch.equal(dst[:, d_blocks], src[:, p_blocks])
        assert not d_work.get_block_ids_with_load_errors()
        st = d_work.get_kv_connector_stats()          # vLLM's per-interval transfer telemetry
        red = st.reduce()
        assert red["loads"] == 1 and red["chunks"] == 4 and red["failed"] == 0 and red["load_ms_max"] > 0
        if not helper:
            assert red["payload_MB"] > 0
        assert d_work.get_kv_connector_stats() is None     # reset after each interval
        agg = SessionKVConnector.build_kv_connector_stats(st.data).aggregate(st)
        assert agg.reduce()["loads"] == 2
        deadline = time.monotonic() + 10
        sending = None
        while time.monotonic() < deadline and not sending:
            sending, _ = _step(p_sched, p_work)
            time.sleep(0.01)
        assert sending == {"p1"}
        assert len(FakeJobs.seen) == 4 and all(v == prompt for _, v in FakeJobs.seen)
    finally:
        p_work.shutdown()
        d_work.shutdown()


def test_cached_prefix_pulls_only_the_suffix():
    FakeJobs.seen.clear()
    src, dst, p_sched, d_sched, p_work, d_work = _pair(_port())
    try:
        prompt, p_blocks = 100, list(range(0, 7))
        d_blocks, suffix = list(range(30, 37)), list(range(34, 37))   # 4 blocks already cached
        _, params = _prefill(p_sched, p_work, "p2", "t2", prompt, p_blocks)
        dreq = _req("d2", prompt, dict(params), status="WAITING_FOR_REMOTE_KVS")
        assert d_sched.get_num_new_matched_tokens(dreq, 64) == (prompt - 64, True)
        d_sched.update_state_after_alloc(dreq, Blocks(d_blocks, suffix), prompt - 64)
        assert _wait_recv(d_sched, d_work, "d2")
        assert torch.equal(dst[:, suffix], src[:, p_blocks[4:]])
        assert dst[:, d_blocks[:4]].abs().sum() == 0
        assert [ids for ids, _ in FakeJobs.seen] == [(4, 5), (6,)]
        assert all(v == prompt - 64 for _, v in FakeJobs.seen)
    finally:
        p_work.shutdown()
        d_work.shutdown()


class SlidingWindowSpec:          # the name vLLM's sliding-window KV-cache spec has
    def __init__(self, window):
        self.sliding_window, self.block_size = window, BS


class FullAttentionSpec(SlidingWindowSpec):
    pass


def _groups(*specs):
    return NS(kv_cache_groups=[NS(kv_cache_spec=s) for s in specs])


def test_sliding_window_pulls_only_the_blocks_in_the_window():
    FakeJobs.seen.clear()
    port = _port()
    src, dst, p_sched, _, p_work, d_work = _pair(port)
    # a 40-token window over 16-token blocks: the last ceil(40/16) + 1 = 4 blocks
    d_sched = FakeJobs(_vllm_config(False, port), KVConnectorRole.SCHEDULER, _groups(SlidingWindowSpec(40)))
    try:
        prompt, p_blocks, d_blocks = 100, list(range(0, 7)), list(range(30, 37))
        _, params = _prefill(p_sched, p_work, "p5", "t5", prompt, p_blocks)
        dreq = _req("d5", prompt, dict(params), status="WAITING_FOR_REMOTE_KVS")
        assert d_sched.get_num_new_matched_tokens(dreq, 0) == (prompt, True)
        d_sched.update_state_after_alloc(dreq, Blocks(d_blocks, d_blocks), prompt)
        assert _wait_recv(d_sched, d_work, "d5")
        assert torch.equal(dst[:, d_blocks[3:]], src[:, p_blocks[3:]])
        assert dst[:, d_blocks[:3]].abs().sum() == 0            # out of the window: not sent
        assert [ids for ids, _ in FakeJobs.seen] == [(3, 4), (5, 6)]
        assert all(v == prompt - 3 * BS for _, v in FakeJobs.seen)
    finally:
        p_work.shutdown()
        d_work.shutdown()


def test_decode_finds_the_producer_through_the_bootstrap_service():
    from kvserve_b200.session.bootstrap import BootstrapClient, Registry, serve
    FakeJobs.seen.clear()
    reg = Registry()
    server, thread = serve("127.0.0.1", _port(), reg)
    url = f"http://127.0.0.1:{server.config.port}"
    port = _port()

    def cfg(producer):
        c = _vllm_config(producer, port)
        c.kv_transfer_config.kv_connector_extra_config.update(bootstrap_url=url, engine_id="prefill-A")
        return c
    src = torch.randn(2, NB, BS, 2, 64).to(torch.bfloat16)
    dst = torch.zeros_like(src)
    p_sched, d_sched = FakeJobs(cfg(True), KVConnectorRole.SCHEDULER), FakeJobs(cfg(False), KVConnectorRole.SCHEDULER)
    p_work, d_work = FakeJobs(cfg(True), KVConnectorRole.WORKER), FakeJobs(cfg(False), KVConnectorRole.WORKER)
    p_work.register_kv_caches({"model.layers.0.self_attn.attn": src})
    d_work.register_kv_caches({"model.layers.0.self_attn.attn": dst})
    try:
        assert reg.query("prefill-A", 0)["endpoint"] == f"tcp://127.0.0.1:{port}"
        prompt, p_blocks, d_blocks = 40, [1, 2, 3], [20, 21, 22]
        _, params = _prefill(p_sched, p_work, "p6", "t6", prompt, p_blocks)
        assert params["remote_engine_id"] == "prefill-A"
        params = dict(params, remote_port=1)          # a wrong direct address: only the registry finds P
        dreq = _req("d6", prompt, params, status="WAITING_FOR_REMOTE_KVS")
        assert d_sched.get_num_new_matched_tokens(dreq, 0) == (prompt, True)
        d_sched.update_state_after_alloc(dreq, Blocks(d_blocks, d_blocks), prompt)
        assert _wait_recv(d_sched, d_work, "d6")
        assert torch.equal(dst[:, d_blocks], src[:, p_blocks])
        p_work.shutdown()                               # rank 0 of the engine leaves the registry
        assert BootstrapClient(url).endpoint("prefill-A", 0) is None
    finally:
        p_work.shutdown()
        d_work.shutdown()
        server.should_exit = True
        thread.join(10)


def test_data_parallel_replicas_register_as_their_own_engines():
    c = _vllm_config(True, _port())
    c.kv_transfer_config.kv_connector_extra_config["engine_id"] = "prefill-A"
    assert FakeJobs(c, KVConnectorRole.SCHEDULER)._engine_id == "prefill-A"
    c.parallel_config = NS(tensor_parallel_size=1, data_parallel_size=2, data_parallel_rank=1)
    assert FakeJobs(c, KVConnectorRole.SCHEDULER)._engine_id == "prefill-A/dp1"
    from kvserve_b200.session.bootstrap import BootstrapClient, serve
    server, thread = serve("127.0.0.1", _port())
    try:
        cl = BootstrapClient(f"http://127.0.0.1:{server.config.port}")
        cl.register("prefill-A/dp1", 1, "tcp://h:2", 2)
        assert cl.endpoint("prefill-A/dp1", 1) == "tcp://h:2" and cl.endpoint("prefill-A/dp0", 1) is None
        assert cl.unregister("prefill-A/dp1") == 1 and cl.endpoint("prefill-A/dp1", 1) is None
    finally:
        server.should_exit = True
        thread.join(10)


def test_window_and_group_rules():
    blocks = SessionKVConnector.sliding_window_blocks
    assert blocks(None) == 0 and blocks(_groups()) == 0
    assert blocks(_groups(SlidingWindowSpec(4096))) == 257
    assert blocks(_groups(SlidingWindowSpec(48))) == 4
    # a full-attention spec that carries a window keeps every block
    assert blocks(_groups(FullAttentionSpec(4096))) == 0
    with pytest.raises(ValueError, match="one KV-cache group"):
        blocks(_groups(FullAttentionSpec(None), SlidingWindowSpec(4096)))


@pytest.mark.parametrize("helper", [False, True], ids=["service-thread", "helper-process"])
def test_unknown_transfer_reports_load_errors(helper):
    src, dst, p_sched, d_sched, p_work, d_work = _pair(_port(), helper)
    try:
        params = {"do_remote_prefill": True, "transfer_id": "nope", "remote_host": "127.0.0.1",
                  "remote_port": p_sched._port}
        dreq = _req("d3", 40, params, status="WAITING_FOR_REMOTE_KVS")
        assert d_sched.get_num_new_matched_tokens(dreq, 0) == (40, True)
        d_sched.update_state_after_alloc(dreq, Blocks([5, 6, 7], [5, 6, 7]), 40)
        assert _wait_recv(d_sched, d_work, "d3")
        assert d_work.get_block_ids_with_load_errors() == {5, 6, 7}
        # a request without router parameters is not the connector's
        assert d_sched.get_num_new_matched_tokens(_req("d4", 40, None), 0) == (0, False)
        # an aborted prefill frees its blocks at once and withdraws its send
        req = _req("p4", 40, {"do_remote_decode": True, "transfer_id": "x"}, status="FINISHED_ABORTED")
        p_sched.update_state_after_alloc(req, Blocks([1, 2, 3], [1, 2, 3]), 0)
        _step(p_sched, p_work, so=_sched_out([("p4", [1, 2, 3], 40)]))
        assert p_sched.request_finished(req, [1, 2, 3]) == (False, None)
        meta = p_sched.build_connector_meta(_sched_out())
        assert meta.cancels == ["x"] and not meta.sends
        # a prefill still in progress is not sent before its last chunk
        req5 = _req("p5", 64, {"do_remote_decode": True, "transfer_id": "y"})
        p_sched.update_state_after_alloc(req5, Blocks([8, 9], [8, 9]), 0)
        assert not p_sched.build_connector_meta(_sched_out([("p5", [8, 9], 32)])).sends
    finally:
        p_work.shutdown()
        d_work.shutdown()


class FakeHeadJobs(SessionKVConnector):
    """Like :class:`FakeJobs`, but each session copies only its KV-head
    range (the copy named by the transfer id) — the GPU jobs bind one
    runtime per copy to the same head slices."""
    arena: dict = {}

    def make_encode_job(self, caches):
        cache = next(iter(caches.values()))
        copies = dict(self._copies)
        self._per_chunk = PER_CHUNK

        def enc(session, pull):
            c = copies[self.copy_key(session.transfer_id)]
            ids = session.local_block_ids[0][pull.chunk_id * PER_CHUNK:(pull.chunk_id + 1) * PER_CHUNK]
            FakeHeadJobs.arena[(session.transfer_id, pull.slot_id)] = \
                cache[:, ids, :, c.src_head:c.src_head + c.heads].clone()
            return 1, 1
        return enc

    def make_decode_job(self, caches):
        cache = next(iter(caches.values()))
        copies = dict(self._copies)
        self._per_chunk = PER_CHUNK

        def dec(session, slot, ready):
            c = copies[self.copy_key(session.transfer_id)]
            ids = session.block_ids[0][ready.chunk_id * PER_CHUNK:(ready.chunk_id + 1) * PER_CHUNK]
            cache[:, ids, :, c.dst_head:c.dst_head + c.heads] = FakeHeadJobs.arena[(session.transfer_id,
                                                                                     slot.slot_id)]
        return dec, 1 << 20, b""


def _tp_config(producer, port, tp, p_tp, d_tp):
    cfgs = _vllm_config(producer, port)
    cfgs.parallel_config = NS(tensor_parallel_size=tp)
    cfgs.kv_transfer_config.kv_connector_extra_config.update(prefill_tp_size=p_tp, decode_tp_size=d_tp,
                                                             num_kv_heads=4)
    return cfgs


def test_heterogeneous_tp_pulls_each_head_range_from_its_holder():
    """Prefill TP 1 (4 KV heads) -> decode TP 2 (2 heads per rank): each
    decode rank opens one session for its half of the heads; the prefill
    rank serves both and reports the request sent after both end."""
    port = _port()
    src = torch.randn(2, NB, BS, 4, 64).to(torch.bfloat16)
    dst = [torch.zeros(2, NB, BS, 2, 64, dtype=torch.bfloat16) for _ in range(2)]
    p_sched = FakeHeadJobs(_tp_config(True, port, 1, 1, 2), KVConnectorRole.SCHEDULER)
    p_work = FakeHeadJobs(_tp_config(True, port, 1, 1, 2), KVConnectorRole.WORKER)
    d_sched, d_work = [], []
    for rank in range(2):
        d_sched.append(FakeHeadJobs(_tp_config(False, port, 2, 1, 2), KVConnectorRole.SCHEDULER))
        w = FakeHeadJobs(_tp_config(False, port, 2, 1, 2), KVConnectorRole.WORKER)
        w._tp_rank = rank
        d_work.append(w)
    try:
        p_work.register_kv_caches({"model.layers.0.self_attn.attn": src})
        for w, d in zip(d_work, dst):
            w.register_kv_caches({"model.layers.0.self_attn.attn": d})
        assert [k for k, _ in p_work._copies] == ["0.0", "1.0"]
        assert [(c.src_rank, c.src_head, c.heads) for _, c in d_work[1]._copies] == [(0, 2, 2)]
        prompt, p_blocks, d_blocks = 100, list(range(0, 7)), list(range(10, 17))
        delay, params = _prefill(p_sched, p_work, "p1", "t1", prompt, p_blocks)
        assert delay and params["remote_tp_size"] == 1
        for rank in range(2):
            dreq = _req("d1", prompt, dict(params), status="WAITING_FOR_REMOTE_KVS")
            assert d_sched[rank].get_num_new_matched_tokens(dreq, 0) == (prompt, True)
            d_sched[rank].update_state_after_alloc(dreq, Blocks(d_blocks, d_blocks), prompt)
        for rank in range(2):
            assert _wait_recv(d_sched[rank], d_work[rank], "d1")
            assert torch.equal(dst[rank][:, d_blocks], src[:, p_blocks, :, 2 * rank:2 * rank + 2])
        deadline = time.monotonic() + 10
        sending = None
        while time.monotonic() < deadline and not sending:
            sending, _ = _step(p_sched, p_work)
            time.sleep(0.01)
        assert sending == {"p1"}
        # a decode request from a prefill engine of another TP size is computed locally
        other = dict(params, remote_tp_size=4, do_remote_prefill=True)
        assert d_sched[0].get_num_new_matched_tokens(_req("d9", prompt, other), 0) == (0, False)
    finally:
        p_work.shutdown()
        for w in d_work:
            w.shutdown()


@pytest.mark.parametrize("inline", [False, True], ids=["shared-arena", "inline"])
def test_real_runtime_pull_on_cpu_engines(inline):
    """The connector with its own jobs (no fakes) on CPU caches: the CPU
    runtime encodes each pulled chunk (Hadamard + 4-bit) into the consumer's
    shared-memory slot (or inline in the reply) and decodes it into the
    request's blocks; the loaded KV is the compressed reconstruction."""
    port = _port()
    comp = {"enable-compression-pipeline": True, "pipeline": ["transformer", "quantizer"],
            "logical_blocks_per_chunk": PER_CHUNK, "high_key_num_levels": 16, "low_key_num_levels": 16,
            "high_value_num_levels": 16, "low_value_num_levels": 16}

    def cfg(producer):
        c = _vllm_config(producer, port)
        c.kv_transfer_config.kv_connector_extra_config.update(compression=comp, inline_payloads=inline)
        return c
    g = torch.Generator().manual_seed(4)
    src = torch.randn(2, NB, BS, 2, 128, generator=g).to(torch.bfloat16)
    dst = torch.zeros_like(src)
    p_sched, p_work = SessionKVConnector(cfg(True), KVConnectorRole.SCHEDULER), \
        SessionKVConnector(cfg(True), KVConnectorRole.WORKER)
    d_sched, d_work = SessionKVConnector(cfg(False), KVConnectorRole.SCHEDULER), \
        SessionKVConnector(cfg(False), KVConnectorRole.WORKER)
    try:
        p_work.register_kv_caches({"model.layers.0.self_attn.attn": src})
        d_work.register_kv_caches({"model.layers.0.self_attn.attn": dst})
        prompt, p_blocks, d_blocks = 100, list(range(0, 7)), list(range(20, 27))
        _, params = _prefill(p_sched, p_work, "p1", "t1", prompt, p_blocks)
        dreq = _req("d1", prompt, dict(params), status="WAITING_FOR_REMOTE_KVS")
        assert d_sched.get_num_new_matched_tokens(dreq, 0) == (prompt, True)
        d_sched.update_state_after_alloc(dreq, Blocks(d_blocks, d_blocks), prompt)
        assert _wait_recv(d_sched, d_work, "d1")
        assert not d_work.get_block_ids_with_load_errors()
        a = src[:, p_blocks].float().reshape(2, -1, 2, 128)[:, :prompt]
        b = dst[:, d_blocks].float().reshape(2, -1, 2, 128)[:, :prompt]
        assert ((a - b).norm() / a.norm()) < 0.15
        assert dst[:, d_blocks].float().reshape(2, -1, 2, 128)[:, prompt:].abs().sum() == 0
    finally:
        p_work.shutdown()
        d_work.shutdown()
