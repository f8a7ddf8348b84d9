"""The push connector's whole worker data path on CPUs: a producer process
gathers a request's blocks layer by layer (``save_kv_layer``), stacks,
compresses and sends them as a CompressedWire bundle in ``wait_for_save``
through the credit transport's gloo data plane; the consumer process's
``start_load_kv`` receives, restores, decompresses and injects them into
the request's blocks of its paged caches.  Raw transfers arrive exactly;
the K4/V4 profile within its quantisation error."""
import os
import socket
from collections import defaultdict, deque
from types import SimpleNamespace as NS

import pytest
import torch
import torch.multiprocessing as mp

L, NB, BS, H, D = 2, 12, 16, 4, 128
SRC, DST, TOKENS = [1, 2, 3, 4], [7, 8, 9, 10], 60
PROFILE = {"enabled": True, "pipeline": ["transformer", "quantizer", "codec"],
           "transformer_config": {"transform_type": "hadamard", "seed": 5},
           "quantizer_config": {"model_name": "synthetic", "hybrid_ratio": 0.0, "high_key_max_value": 15,
                                "high_value_max_value": 15, "low_key_max_value": 15, "low_value_max_value": 15,
                                "axis_key": "channel", "axis_value": "token", "split_type": "head",
                                "num_layers": L, "num_kv_heads": H},
           "codec_config": {"codec_type": "bitpack", "bitpack_bits": 4}}


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _connector(producer, port, compression):
    from kvserve_b200.connector.compressed_kv_connector import (CompressedKVConnector,
                                                                CompressedKVConnectorMetadata)
    c = CompressedKVConnector.__new__(CompressedKVConnector)
    c.is_producer = producer
    c._transport = CompressedKVConnector._build_transport(
        NS(is_kv_producer=producer, kv_ip="127.0.0.1", kv_port=port, kv_buffer_size=64 << 20), 0, 0, "gloo")
    c._worker_received_kv, c._layer_buffers = defaultdict(deque), {}
    c._compression_cfg, c._compressor = compression, None
    c._num_kv_heads, c._head_size, c._num_layers = H, D, L
    c._model_name, c._tp_rank, c._tp_size = "synthetic", 0, 1
    c._async_send, c._block_size = False, BS
    c._request_transfer_ids, c._requests_need_load, c.chunked_prefill = {}, {}, {}
    meta = CompressedKVConnectorMetadata()
    meta.add_request("r1", "t1", list(range(TOKENS)), SRC if producer else DST, BS)
    c._connector_metadata = meta
    return c


def _caches(fill):
    g = torch.Generator().manual_seed(8)
    mk = (lambda: torch.randn(2, NB, BS, H, D, generator=g)) if fill else (lambda: torch.zeros(2, NB, BS, H, D))
    return {f"model.layers.{i}.self_attn.attn": mk().to(torch.bfloat16) for i in range(L)}


def _finish(q, role, out, done=None):
    """Report and leave without tearing the transport down: its control
    thread may still be inside a ZeroMQ call, and closing the socket under it
    aborts the process."""
    q.put((role, out))
    if done is not None:
        done.wait(60)          # the consumer may still need this side's replies
    q.close()
    q.join_thread()
    os._exit(0)


def _producer(port, compression, q, done):
    out = {"error": None}
    try:
        c = _connector(True, port, compression)
        for name, kv in _caches(True).items():
            c.save_kv_layer(name, kv, None)
        c.wait_for_save()
        c.shutdown()
    except Exception:  # noqa: BLE001
        import traceback
        out["error"] = traceback.format_exc()
    _finish(q, "producer", out, done)


def _consumer(port, compression, q, done):
    out = {"error": None}
    try:
        c = _connector(False, port, compression)
        caches = _caches(False)
        fc = NS(no_compile_layers={n: NS(kv_cache=t) for n, t in caches.items()}, virtual_engine=0)
        c.start_load_kv(fc)
        src = _caches(True)
        idx_s, idx_d = torch.tensor(SRC), torch.tensor(DST)
        errs = []
        for n in caches:
            a = src[n].index_select(1, idx_s).float()
            b = caches[n].index_select(1, idx_d).float()
            errs.append(float((a - b).norm() / a.norm()))
        out["max_rel_err"] = max(errs)
        out["others_zero"] = all(float(caches[n].index_select(1, torch.tensor([0, 5, 11])).abs().sum()) == 0
                                 for n in caches)
    except Exception:  # noqa: BLE001
        import traceback
        out["error"] = traceback.format_exc()
    _finish(q, "consumer", out)


@pytest.mark.parametrize("compression", [None, PROFILE], ids=["raw", "k4v4"])
def test_push_connector_moves_a_request_over_gloo(compression):
    ctx = mp.get_context("spawn")
    q, done = ctx.Queue(), ctx.Event()
    port = _port()
    procs = [ctx.Process(target=_consumer, args=(port, compression, q, done)),
             ctx.Process(target=_producer, args=(port, compression, q, done))]
    procs[0].start()
    import time
    time.sleep(0.5)
    procs[1].start()
    try:
        res = {}
        for _ in procs:
            role, out = q.get(timeout=120)
            res[role] = out
            if role == "consumer":
                done.set()
    finally:
        done.set()
        for p in procs:
            p.join(30)
            if p.is_alive():
                p.kill()
    for r in res.values():
        assert r["error"] is None, r["error"]
    c = res["consumer"]
    assert c["others_zero"]
    if compression is None:
        assert c["max_rel_err"] == 0.0
    else:
        assert 0.0 < c["max_rel_err"] < 0.15
