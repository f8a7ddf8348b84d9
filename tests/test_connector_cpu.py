"""Connector logic on CPU with a fake transport (no vLLM engine, no GPU)."""
from collections import defaultdict, deque
from types import SimpleNamespace

import pytest
import torch


class FakeTransport:
    def __init__(self, arrivals):
        self.arrivals = deque(arrivals)  # (transfer_id, (names, payload)) delivered one per drain
        self.released = []
        self.expected = []
        self.stats = []
        self.device = torch.device("cpu")
        self.sent = []

    def drain_received(self):
        if not self.arrivals:
            return {}
        nxt = self.arrivals.popleft()
        if nxt is None:
            return {}
        tid, item = nxt
        return {tid: [item]}

    def set_expected_requests(self, ids):
        self.expected.append(list(ids))

    def payload_nbytes(self, p):
        from kvserve_b200.transport.nccl_transport import payload_nbytes
        return payload_nbytes(p)

    def release_received(self, tid, n):
        self.released.append((tid, n))

    def record_stat(self, row):
        self.stats.append(row)

    def send(self, tid, names, t):
        self.sent.append(("raw", tid, names, t))

    def send_bundle(self, tid, names, meta, body, aux):
        self.sent.append(("bundle", tid, names, meta, body, aux))

    def wait_for_sent(self):
        pass


def _bare(is_producer, transport, compression=None):
    from kvserve_b200.connector.compressed_kv_connector import CompressedKVConnector
    c = CompressedKVConnector.__new__(CompressedKVConnector)
    c.is_producer = is_producer
    c._transport = transport
    c._worker_received_kv = defaultdict(deque)
    c._layer_buffers = {}
    c._compression_cfg = compression
    c._compressor = None
    c._num_kv_heads, c._head_size, c._num_layers = 4, 128, 2
    c._model_name, c._tp_rank, c._tp_size = "synthetic", 0, 1
    c._async_send = False
    c._block_size = 16
    c._request_transfer_ids = {}
    c._requests_need_load = {}
    c.chunked_prefill = {}
    return c


def _meta(*tids):
    from kvserve_b200.connector.compressed_kv_connector import CompressedKVConnectorMetadata
    m = CompressedKVConnectorMetadata()
    for t in tids:
        m.add_request("req-" + t, t, list(range(20)), [0, 1], 16)
    return m


def test_consumer_consumes_out_of_order_and_releases_credit(monkeypatch):
    # "b" (scheduled second) arrives first and must not wait behind "a"
    tr = FakeTransport([None, ("b", (["l0"], torch.zeros(1, 2, 2, 16, 4, 128))), None,
                        ("a", (["l0"], torch.ones(1, 2, 2, 16, 4, 128)))])
    c = _bare(False, tr)
    c._get_connector_metadata = lambda: _meta("a", "b")
    injected = []
    c.inject = lambda fc, names, stacked, req: injected.append((req.transfer_id, float(stacked.sum())))
    c.start_load_kv(SimpleNamespace())
    assert [i[0] for i in injected] == ["b", "a"]
    assert [r[0] for r in tr.released] == ["b", "a"] and all(n > 0 for _, n in tr.released)
    assert tr.expected[0] == ["a", "b"] and tr.expected[-1] == []


def test_consumer_fails_fast_on_failure_sentinel():
    tr = FakeTransport([("a", ([], None))])
    c = _bare(False, tr)
    c._get_connector_metadata = lambda: _meta("a")
    c.inject = lambda *a: None
    with pytest.raises(RuntimeError, match="transport failed"):
        c.start_load_kv(SimpleNamespace())


def test_consumer_times_out(monkeypatch):
    import kvserve_b200.connector.compressed_kv_connector as mod
    monkeypatch.setattr(mod, "LOAD_TIMEOUT_S", 0.1)
    tr = FakeTransport([])
    c = _bare(False, tr)
    c._get_connector_metadata = lambda: _meta("x")
    with pytest.raises(TimeoutError):
        c.start_load_kv(SimpleNamespace())
    assert any(s.get("kind") == "timeout" for s in tr.stats)


def test_producer_compressed_bundle_round_trip():
    from test_compression_cpu import CFG0, synthetic_kv
    tr = FakeTransport([])
    prod = _bare(True, tr, compression=CFG0)
    kv = synthetic_kv()  # [L, 2, 1, 256, 4, 128]
    stacked = kv.view(2, 2, 16, 16, 4, 128)
    prod.send_stacked("req-1", "t-1", ["l0", "l1"], stacked)
    kind, tid, names, meta, body, aux = tr.sent[0]
    assert kind == "bundle" and names[0] == "__compressed__"
    cons = _bare(False, FakeTransport([("t-1", (names, {"__bundle__": True, "meta": meta, "body_chunks": body,
                                                        "aux_tensors": aux}))]), compression=CFG0)
    cons._get_connector_metadata = lambda: _meta("t-1")
    got = []
    cons.inject = lambda fc, n, s, req: got.append((n, s))
    cons.start_load_kv(SimpleNamespace())
    names_out, restored = got[0]
    assert names_out == ["l0", "l1"] and restored.shape == stacked.shape
    assert ((restored.float() - stacked.float()).norm() / stacked.float().norm()) < 0.2


def test_scheduler_claims_prompt_minus_one():
    c = _bare(False, FakeTransport([]))
    req = SimpleNamespace(prompt_token_ids=list(range(100)), request_id="r", kv_transfer_params={"transfer_id": "T"})
    assert c.get_num_new_matched_tokens(req, 0) == (99, False)
    assert c.get_num_new_matched_tokens(req, 99) == (0, False)
    c.update_state_after_alloc(req, SimpleNamespace(get_block_ids=lambda: [[3, 4]]), 99)
    assert c._resolve_transfer_id("r") == "T" and "r" in c._requests_need_load
    p = _bare(True, FakeTransport([]))
    assert p.get_num_new_matched_tokens(req, 0) == (0, False)


def test_worker_memory_plan_matches_runtime_plan():
    from types import SimpleNamespace

    import torch
    from kvserve_b200.compression.runtime import CompressionConfig, build_memory_plan
    from kvserve_b200.connector.memory_plan import (KVConnectorWorkerMemoryPlan, adjusted_utilization,
                                                    cache_specs_from_vllm, layer_index_of, plan_worker_memory)
    specs = {f"model.layers.{i}.self_attn.attn": SimpleNamespace(block_size=16, num_kv_heads=8, head_size=128,
                                                                  dtype=torch.bfloat16) for i in range(4)}
    assert layer_index_of("model.layers.12.self_attn.attn") == 12
    assert plan_worker_memory({}, specs) == KVConnectorWorkerMemoryPlan()
    extra = {"compression": {"enable-compression-pipeline": True, "slot_count": 3}}
    plan = plan_worker_memory(extra, specs)
    ref = build_memory_plan(CompressionConfig.from_extra_config(extra), cache_specs_from_vllm(specs))
    assert plan.reserved_bytes == ref.reserved_bytes > 0
    assert plan.connector_data.slot_bytes == ref.slot_bytes
    u = adjusted_utilization(100 * 2 ** 30, 0.9, plan)
    assert abs(u * 100 * 2 ** 30 - (0.9 * 100 * 2 ** 30 - plan.reserved_bytes)) < 1.0


def test_service_aware_engine_library_and_selection():
    """Engine profiles -> library: more bits are more accurate and less
    compressed; the controller's choice respects the accuracy requirement."""
    from kvserve_b200.compression.controller.online import OnlineController
    from kvserve_b200.engine.serving import ENGINE_PROFILES, engine_library
    from kvserve_b200.engine.transfer import KVTransfer

    class _Eng:
        pass
    eng = _Eng()
    eng.cfg = type("C", (), {"name": "tiny"})()
    eng.xfers = {n: KVTransfer(p, 2, 4, 4, 128, 0, 1, "cpu", 256) for n, p in ENGINE_PROFILES.items()}
    speeds = {"k8v8": 9e5, "k4v4": 6e5, "k4v2": 5e5, "k2v2": 4e5}
    lib = engine_library(eng, 256, speeds)
    prof = {p.profile_id: p for b in lib.accuracy_buckets for p in
            (lib.get_profile(d["profile_id"]) for d in b["pareto_profiles"])}
    import math
    from kvserve_b200.engine.serving import profile_accuracy
    acc = {n: profile_accuracy(ENGINE_PROFILES[n], 4, 128) for n in speeds}
    assert acc["k8v8"] > acc["k4v4"] > acc["k4v2"] > acc["k2v2"] > 0.1
    cr = {n: eng.xfers[n].raw_bytes(256) / eng.xfers[n].payload_bytes(256) for n in speeds}
    assert cr["k2v2"] > cr["k4v2"] > cr["k4v4"] > cr["k8v8"] > 1.5
    assert prof and all(math.isfinite(p.compression_ratio) for p in prof.values())
    from kvserve_b200.engine.serving import bucket_requirement
    ctl = OnlineController(lib, epsilon=0.0)
    for need in (0.2, 0.5, acc["k4v4"] - 1e-4, acc["k8v8"] - 1e-4):
        p, info = ctl.select_profile(2e9, 3125.0, 100.0, 1e9, bucket_requirement(lib, need))
        assert p is not None and p.accuracy >= need, (need, p, info)
    assert ctl.select_profile(2e9, 3125.0, 100.0, 1e9, bucket_requirement(lib, 0.2))[0].profile_id == "k2v2"
    assert bucket_requirement(lib, 0.9999) is None    # nothing compressed is that accurate


def test_inject_on_vllm_022_caches_both_layouts():
    """vLLM 0.22 keeps one cache tensor per layer and has no virtual_engine;
    FlashInfer (its B200 default) stores [blocks, 2, ...].  The wire is always
    [2, blocks, ...]; older list-per-virtual-engine caches still work."""
    from types import SimpleNamespace
    from kvserve_b200.connector.compressed_kv_connector import CompressedKVConnector, ReqMeta
    fa = torch.zeros(2, 6, 4, 2, 8)
    fi = torch.zeros(6, 2, 4, 2, 8)
    old = torch.zeros(2, 6, 4, 2, 8)
    layers = {"a": SimpleNamespace(kv_cache=fa), "b": SimpleNamespace(kv_cache=fi),
              "c": SimpleNamespace(kv_cache=[old]), "d": SimpleNamespace(kv_cache=torch.tensor([]))}
    ctx = SimpleNamespace(no_compile_layers=layers)           # no virtual_engine attribute
    stacked = torch.randn(4, 2, 2, 4, 2, 8)
    req = ReqMeta("r", "t", list(range(8)), [3, 1], torch.arange(8))
    CompressedKVConnector.inject(ctx, ["a", "b", "c", "d"], stacked, req)
    assert torch.equal(fa[:, [3, 1]], stacked[0])
    assert torch.equal(fi[[3, 1]], stacked[1].transpose(0, 1))
    assert torch.equal(old[:, [3, 1]], stacked[2])


def test_example_configs_build_and_name_real_connectors():
    """The examples' vLLM configurations build and point at importable
    connector classes."""
    import importlib
    import os
    import sys
    pytest.importorskip("vllm")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "examples"))
    try:
        ex = importlib.import_module("vllm_connectors")
        cfgs = [ex.push_config("kv_producer"), ex.push_config("kv_consumer", data_plane="ipc"),
                ex.pull_config("kv_producer"), ex.pull_config("kv_consumer", prefill_tp=1, decode_tp=2),
                ex.store_config("/tmp/kvs-store-example", disk_bytes=1 << 30)]
        for c in cfgs:
            cls = getattr(importlib.import_module(c.kv_connector_module_path), c.kv_connector)
            assert cls.__name__ == c.kv_connector
        assert cfgs[3].kv_connector_extra_config["decode_tp_size"] == 2
        boot = ex.pull_config("kv_producer", bootstrap_url="http://127.0.0.1:8998", engine_id="prefill-0")
        assert boot.kv_connector_extra_config["bootstrap_url"] == "http://127.0.0.1:8998"
        assert boot.kv_connector_extra_config["engine_id"] == "prefill-0"
        p = ex.pull_prefill_params("t-1")
        assert p.max_tokens == 1 and p.extra_args["kv_transfer_params"]["do_remote_decode"]
        with pytest.raises(ValueError):
            ex.push_config("kv_both")
    finally:
        sys.path.remove(os.path.join(root, "examples"))
