"""The transport's GPU data planes on real GPUs.

* CUDA IPC (no NCCL on the KV path): a producer process and a consumer
  process (both on GPU 0, or on GPUs 0 and 1 when two are visible) exchange
  raw and bundle payloads; the consumer's pool grants ranges, the producer's
  copy engine writes them, ``DONE`` publishes them.
* NCCL (the reference's own data plane, kvserve_v1/transport/
  nccl_transport.py:312-445, 600-725): the same exchange over a two-rank NCCL
  communicator, which needs two GPUs (skipped with one).

Checked: the bytes arrive intact, credit-released ranges are reused, and a
payload larger than the receive budget (admitted into an empty buffer, the
oversize rule) still travels.
"""
import multiprocessing as mp
import os
import socket
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _payload(i: int, n: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(i)
    return torch.randint(0, 255, (n,), generator=g, dtype=torch.uint8)


def _consumer(port, dev, q, expect, plane="ipc"):
    torch.cuda.set_device(dev)
    from kvserve_b200.transport.nccl_transport import NcclTransport
    t = NcclTransport(False, "127.0.0.1", port, local_rank=dev, data_plane=plane, recv_buffer_size=4 << 20)
    got = {}
    deadline = time.time() + 120
    while len(got) < expect and time.time() < deadline:
        for rid, items in t.drain_received().items():
            for names, payload in items:
                if payload is None:
                    got[rid] = None
                    continue
                if isinstance(payload, dict):
                    data = [x.cpu().clone() for x in payload["body_chunks"] + payload["aux_tensors"]]
                    got[rid] = ("bundle", names, payload["meta"], data)
                else:
                    got[rid] = ("raw", names, payload.cpu().clone())
                t.release_received(rid, t.payload_nbytes(payload))
        time.sleep(0.005)
    pool = getattr(t.plane, "_pool", None)
    q.put({"got": got, "free": pool.free_bytes() if pool else 0, "cap": pool.size if pool else 0})
    time.sleep(0.5)
    t.close()


def _producer(port, dev, q, plane="ipc"):
    torch.cuda.set_device(dev)
    from kvserve_b200.transport.nccl_transport import NcclTransport
    t = NcclTransport(True, "127.0.0.1", port, local_rank=dev, data_plane=plane, control_timeout_s=30)
    for i in range(6):   # 6 x 1.5 MiB through a 4 MiB pool: ranges must be reused
        t.send(f"r{i}", ["l0"], _payload(i, 3 << 19).cuda())
    t.send_bundle("b0", ["__compressed__", "l0"], {"k": 1}, [_payload(10, 1000).cuda(), _payload(11, 77).cuda()],
                  [_payload(12, 40).cuda()])
    t.send("big", ["l0"], _payload(20, 6 << 20).cuda())   # larger than the whole pool
    q.put(t.wait_for_sent(timeout=120))
    time.sleep(1.0)
    t.close()


@pytest.mark.parametrize("plane", ["ipc", pytest.param("nccl", marks=pytest.mark.multigpu)])
def test_data_plane_moves_payloads(plane):
    if plane == "nccl" and torch.cuda.device_count() < 2:
        pytest.skip("the NCCL data plane needs two GPUs")
    if plane == "nccl":
        os.environ["NCCL_NVLS_ENABLE"] = "0"
    devs = (0, 1) if torch.cuda.device_count() > 1 else (0, 0)
    ctx = mp.get_context("spawn")
    port = _free_port()
    qc, qp = ctx.Queue(), ctx.Queue()
    c = ctx.Process(target=_consumer, args=(port, devs[1], qc, 8, plane))
    p = ctx.Process(target=_producer, args=(port, devs[0], qp, plane))
    c.start()
    time.sleep(1.0)
    p.start()
    res = qc.get(timeout=240)
    ok = qp.get(timeout=240)
    for proc in (p, c):
        proc.join(30)
        if proc.is_alive():
            proc.kill()
    got = res["got"]
    assert ok and len(got) == 8
    for i in range(6):
        kind, names, data = got[f"r{i}"]
        assert kind == "raw" and names == ["l0"] and torch.equal(data, _payload(i, 3 << 19))
    kind, names, meta, data = got["b0"]
    assert kind == "bundle" and meta == {"k": 1}
    for d, seed, n in zip(data, (10, 11, 12), (1000, 77, 40)):
        assert torch.equal(d, _payload(seed, n))
    assert torch.equal(got["big"][2], _payload(20, 6 << 20))
    if plane == "ipc":
        assert res["free"] == res["cap"]      # every granted range came back
