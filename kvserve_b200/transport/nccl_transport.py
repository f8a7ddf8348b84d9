"""Point-to-point KV transport with ZMQ control and receiver credits — the
API and message protocol of kvserve_v1/transport/nccl_transport.py:83-768,
re-implemented (own threads, own data-plane abstraction).

Control (ZMQ DEALER -> ROUTER on ``port + channel_rank``, msgpack):
``INIT {unique_id | gloo rendezvous}``, ``PUT {request_id, layer_names, shape,
dtype}``, ``PUT_BUNDLE {request_id, layer_names, meta, body_specs,
aux_specs}``; the consumer answers ``b"0"`` (ACK, then the data follows),
``b"1"`` (out of memory / not initialised: the transfer fails fast via the
``FAILED_PAYLOAD`` sentinel) or ``b"2"`` (RETRY: no staging credit now — the
producer rotates the item behind others while keeping per-request order).

Credits: the consumer admits a payload while reserved + size <= capacity; a
single oversize payload is admitted into an empty buffer; one "priority"
payload of a currently expected request may exceed the budget.  Credit is
returned by ``release_received`` after the KV has been injected.

Data plane: ``"nccl"`` (2-rank NCCL communicator, dedicated CUDA streams,
completion threads retire events in order) or ``"gloo"`` (CPU tensors over
a 2-rank gloo group; used for CPU runs and failure tests).
Stats rows go to ``KVSERVE_TRANSPORT_STATS_PATH`` as JSONL.
"""
from __future__ import annotations

import datetime
import json
import logging
import math
import os
import threading
import time
from collections import defaultdict, deque
from typing import Any, Optional

import msgpack
import torch
import zmq

from .faults import FaultInjector

log = logging.getLogger("kvserve_b200.transport")

ACK_OK = b"0"
ACK_OOM = b"1"
ACK_RETRY = b"2"
_RETRY = object()
FAILED_PAYLOAD: Any = None
FAILED_LAYER_NAMES: list = []


def tensor_nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


def spec_nbytes(spec: dict) -> int:
    return math.prod(spec["shape"]) * torch.empty((), dtype=getattr(torch, spec["dtype"])).element_size()


def payload_nbytes(payload: Any) -> int:
    if isinstance(payload, torch.Tensor):
        return tensor_nbytes(payload)
    if isinstance(payload, dict) and payload.get("__bundle__"):
        return sum(tensor_nbytes(t) for t in payload["body_chunks"] + payload["aux_tensors"])
    return 0


def _spec(t: torch.Tensor) -> dict:
    return {"shape": list(t.shape), "dtype": str(t.dtype).replace("torch.", "")}


# ------------------------------------------------------------------ data planes
class _NcclPlane:
    def __init__(self, device: torch.device):
        from .nccl_lib import NcclLib
        self.lib = NcclLib.get()
        self.device = device
        self.comm = 0
        self.stream = torch.cuda.Stream(device=device)

    def producer_init(self) -> dict:
        uid = self.lib.unique_id()
        self._uid = uid
        return {"unique_id": uid}

    def producer_connect(self) -> None:
        with torch.cuda.device(self.device):
            self.comm = self.lib.comm_init(2, self._uid, 0)

    def consumer_connect(self, msg: dict) -> None:
        with torch.cuda.device(self.device):
            self.comm = self.lib.comm_init(2, msg["unique_id"], 1)

    def alloc(self, shape, dtype) -> torch.Tensor:
        return torch.empty(shape, dtype=dtype, device=self.device)

    def send(self, tensors: list, ready: Optional[torch.cuda.Event]):
        with torch.cuda.stream(self.stream):
            if ready is not None:
                self.stream.wait_event(ready)
            start = torch.cuda.Event(enable_timing=True)
            start.record(self.stream)
            for t in tensors:
                if t.numel():
                    self.lib.send(t, 1, self.comm, self.stream.cuda_stream)
            done = torch.cuda.Event(enable_timing=True)
            done.record(self.stream)
        return start, done

    def recv(self, tensors: list):
        with torch.cuda.stream(self.stream):
            start = torch.cuda.Event(enable_timing=True)
            start.record(self.stream)
            for t in tensors:
                if t.numel():
                    self.lib.recv(t, 0, self.comm, self.stream.cuda_stream)
            done = torch.cuda.Event(enable_timing=True)
            done.record(self.stream)
        return start, done

    @staticmethod
    def wait(handle) -> float:
        start, done = handle
        done.synchronize()
        return start.elapsed_time(done) / 1e3

    def close(self) -> None:
        if self.comm:
            self.lib.destroy(self.comm)
            self.comm = 0


class _GlooPlane:
    """2-rank gloo group built from a TCPStore the producer hosts."""

    def __init__(self, host: str, store_port: int, timeout_s: float = 60.0):
        self.host, self.store_port, self.timeout = host, store_port, datetime.timedelta(seconds=timeout_s)
        self.pg = None
        self._tag = 0

    def producer_init(self) -> dict:
        return {"gloo_host": self.host, "gloo_port": self.store_port}

    def _make(self, rank: int, host: str, port: int) -> None:
        import torch.distributed as dist
        store = dist.TCPStore(host, port, 2, rank == 0, timeout=self.timeout, wait_for_workers=False)
        self.pg = dist.ProcessGroupGloo(store, rank, 2, self.timeout)

    def producer_connect(self) -> None:
        self._make(0, self.host, self.store_port)

    def consumer_connect(self, msg: dict) -> None:
        self._make(1, msg["gloo_host"], int(msg["gloo_port"]))

    @staticmethod
    def alloc(shape, dtype) -> torch.Tensor:
        return torch.empty(shape, dtype=dtype)

    def send(self, tensors: list, ready=None):
        t0 = time.perf_counter()
        for t in tensors:
            if t.numel():
                self.pg.send([t.contiguous()], 1, 0).wait()
        return time.perf_counter() - t0

    def recv(self, tensors: list):
        t0 = time.perf_counter()
        for t in tensors:
            if t.numel():
                self.pg.recv([t], 0, 0).wait()
        return time.perf_counter() - t0

    @staticmethod
    def wait(handle) -> float:
        return float(handle)

    def close(self) -> None:
        self.pg = None


# -------------------------------------------------------------------- transport
class NcclTransport:
    def __init__(self, is_sender: bool, host: str, port: int, local_rank: int = 0, channel_rank: int = 0,
                 recv_buffer_size: int = 1_000_000_000, data_plane: str = "nccl",
                 faults: Optional[FaultInjector] = None, control_timeout_s: float = 60.0):
        self.is_sender = is_sender
        self.local_rank, self.channel_rank = local_rank, channel_rank
        self.port = port + channel_rank
        self.plane_kind = data_plane
        self.device = torch.device(f"cuda:{local_rank}") if data_plane == "nccl" else torch.device("cpu")
        self._stats_path = os.environ.get("KVSERVE_TRANSPORT_STATS_PATH")
        self._stats_lock = threading.Lock()
        self.faults = faults or FaultInjector.from_env()
        self._ctx = zmq.Context()
        self._closed = False
        if data_plane == "nccl":
            self.plane = _NcclPlane(self.device)
        elif data_plane == "gloo":
            self.plane = _GlooPlane(host, port + 1000 + channel_rank)
        else:
            raise ValueError("data_plane must be 'nccl' or 'gloo'")
        if is_sender:
            self._sock = self._ctx.socket(zmq.DEALER)
            self._sock.setsockopt(zmq.RCVTIMEO, int(control_timeout_s * 1000))
            self._sock.setsockopt(zmq.LINGER, 0)
            self._sock.connect(f"tcp://{host}:{self.port}")
            init = {"cmd": "INIT", **self.plane.producer_init()}
            self._sock.send(msgpack.dumps(init, use_bin_type=True))
            self.plane.producer_connect()
            self._q_cv = threading.Condition()
            self._queue: deque = deque()
            self._inflight = 0
            self._pending_bytes = 0
            self._done_cv = threading.Condition()
            self._done: deque = deque()
            threading.Thread(target=self._send_completion_loop, daemon=True, name="kvs-send-done").start()
            threading.Thread(target=self._send_loop, daemon=True, name="kvs-send").start()
        else:
            self._sock = self._ctx.socket(zmq.ROUTER)
            self._sock.setsockopt(zmq.LINGER, 0)
            self._sock.bind(f"tcp://*:{self.port}")
            self._lock = threading.Lock()
            self._budget_cv = threading.Condition(self._lock)
            self._capacity = max(1, int(recv_buffer_size))
            self._reserved = 0
            self._expected: set[str] = set()
            self._priority: Optional[str] = None
            self._received: dict[str, deque] = defaultdict(deque)
            self._rdone_cv = threading.Condition()
            self._rdone: deque = deque()
            self._ready = False
            threading.Thread(target=self._recv_completion_loop, daemon=True, name="kvs-recv-done").start()
            threading.Thread(target=self._listen_loop, daemon=True, name="kvs-listen").start()

    # ------------------------------------------------------------ producer
    def _enqueue(self, item: tuple, nbytes: int) -> None:
        with self._q_cv:
            self._pending_bytes += nbytes
            self._queue.append(item + (time.monotonic_ns(), len(self._queue) + self._inflight + 1,
                                       self._pending_bytes, nbytes))
            self._q_cv.notify()

    def _ready_event(self):
        if self.plane_kind != "nccl":
            return None
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        return ev

    def send(self, request_id: str, layer_names: list, stacked_kv: torch.Tensor) -> None:
        assert self.is_sender
        t = stacked_kv.to(self.device).contiguous()
        self._enqueue(("tensor", request_id, list(layer_names), t, self._ready_event()), tensor_nbytes(t))

    def send_bundle(self, request_id: str, layer_names: list, meta: dict, body_chunks: list,
                    aux_tensors: list) -> None:
        assert self.is_sender
        body = [t.to(self.device).contiguous() for t in body_chunks]
        aux = [t.to(self.device).contiguous() for t in aux_tensors]
        self._enqueue(("bundle", request_id, list(layer_names), meta, body, aux, self._ready_event()),
                      sum(tensor_nbytes(t) for t in body + aux))

    def wait_for_sent(self, timeout: Optional[float] = None) -> bool:
        assert self.is_sender
        deadline = None if timeout is None else time.monotonic() + timeout
        with self._q_cv:
            while self._queue or self._inflight:
                left = None if deadline is None else deadline - time.monotonic()
                if left is not None and left <= 0:
                    return False
                self._q_cv.wait(left)
        return True

    def wait_for_below(self, max_pending_bytes: int) -> float:
        assert self.is_sender
        t0 = time.perf_counter()
        with self._q_cv:
            while self._pending_bytes > max_pending_bytes:
                self._q_cv.wait()
        return time.perf_counter() - t0

    def pending_bytes(self) -> int:
        with self._q_cv:
            return self._pending_bytes

    def _finish(self, nbytes: int) -> None:
        with self._q_cv:
            self._pending_bytes -= nbytes
            self._inflight -= 1
            self._q_cv.notify_all()

    def _send_loop(self) -> None:
        while not self._closed:
            with self._q_cv:
                while not self._queue:
                    self._q_cv.wait()
                item = self._queue.popleft()
                self._inflight += 1
            nbytes = int(item[-1])
            try:
                res = self._send_item(item)
                if res is _RETRY:
                    with self._q_cv:
                        self._inflight -= 1
                        idx = next((i for i, q in enumerate(self._queue) if q[1] == item[1]), len(self._queue))
                        self._queue.insert(idx, item)
                        self._q_cv.notify_all()
                    self._record_stat({"direction": "credit_retry", "kind": item[0], "request_id": item[1],
                                       "payload_bytes": nbytes})
                    time.sleep(0.005)
                elif res is None:
                    self._finish(nbytes)
                else:
                    with self._done_cv:
                        self._done.append(res)
                        self._done_cv.notify()
            except Exception as exc:  # logged, item retired
                log.error("send of %s failed: %s", item[1], exc)
                self._finish(nbytes)

    def _send_item(self, item: tuple):
        kind, rid, names = item[0], item[1], item[2]
        enq_ns, depth, queued, nbytes = item[-4:]
        started = time.monotonic_ns()
        if kind == "tensor":
            t, ready = item[3], item[4]
            msg = {"cmd": "PUT", "request_id": rid, "layer_names": names, **_spec(t)}
            tensors, extra = [t], {"kind": "raw"}
        else:
            meta, body, aux, ready = item[3], item[4], item[5], item[6]
            msg = {"cmd": "PUT_BUNDLE", "request_id": rid, "layer_names": names, "meta": meta,
                   "body_specs": [_spec(t) for t in body], "aux_specs": [_spec(t) for t in aux]}
            tensors, extra = body + aux, {"kind": "bundle", "body_tensors": len(body), "aux_tensors": len(aux)}
        t0 = time.perf_counter()
        self._sock.send(msgpack.dumps(msg, use_bin_type=True))
        ack = self._sock.recv()
        ack_s = time.perf_counter() - t0
        if ack == ACK_RETRY:
            return _RETRY
        if ack != ACK_OK:
            log.error("consumer refused %s (ack=%r)", rid, ack)
            return None
        handle = self.plane.send(tensors, ready)
        row = {"direction": "send", "request_id": rid, "payload_bytes": nbytes, "queue_depth_at_submit": depth,
               "queued_bytes_at_submit": queued, "queue_wait_s": (started - enq_ns) / 1e9, "ack_s": ack_s,
               "_enq": enq_ns, **extra}
        return handle, row, nbytes, tensors

    def _send_completion_loop(self) -> None:
        while not self._closed:
            with self._done_cv:
                while not self._done:
                    self._done_cv.wait()
                handle, row, nbytes, keep = self._done.popleft()
            try:
                row["nccl_s"] = self.plane.wait(handle)
                row["total_s"] = (time.monotonic_ns() - row.pop("_enq")) / 1e9
                self._record_stat(row)
            except Exception as exc:
                log.error("send completion of %s failed: %s", row.get("request_id"), exc)
            finally:
                del keep
                self._finish(nbytes)

    # ------------------------------------------------------------ consumer
    def drain_received(self) -> dict[str, list]:
        assert not self.is_sender
        with self._lock:
            out = {k: list(v) for k, v in self._received.items() if v}
            self._received.clear()
        return out

    @staticmethod
    def payload_nbytes(payload: Any) -> int:
        return payload_nbytes(payload)

    def release_received(self, request_id: str, payload_bytes: int) -> None:
        assert not self.is_sender
        if payload_bytes <= 0:
            return
        with self._budget_cv:
            before = self._reserved
            self._reserved = max(0, self._reserved - int(payload_bytes))
            if request_id == self._priority:
                self._priority = None
            after = self._reserved
            self._budget_cv.notify_all()
        self._record_stat({"direction": "recv_credit_release", "kind": "release", "request_id": request_id,
                           "payload_bytes": int(payload_bytes), "reserved_before_bytes": before,
                           "reserved_after_bytes": after, "capacity_bytes": self._capacity})

    def set_expected_requests(self, request_ids: list) -> None:
        with self._budget_cv:
            self._expected = set(request_ids)
            self._budget_cv.notify_all()

    def reserved_bytes(self) -> int:
        with self._lock:
            return self._reserved

    def _reserve(self, rid: str, nbytes: int, wait: bool = False) -> bool:
        t0 = time.perf_counter()
        if self.faults.refuse_credit(rid):
            return False
        with self._budget_cv:
            blocked = self._reserved > 0 and self._reserved + nbytes > self._capacity
            while self._reserved > 0 and self._reserved + nbytes > self._capacity:
                if rid in self._expected and self._priority is None:
                    self._priority = rid
                    break
                if not wait:
                    return False
                self._budget_cv.wait()
            before = self._reserved
            self._reserved += nbytes
            after = self._reserved
        self._record_stat({"direction": "recv_credit", "kind": "reserve", "request_id": rid, "payload_bytes": nbytes,
                           "blocked": blocked, "wait_s": time.perf_counter() - t0, "reserved_before_bytes": before,
                           "reserved_after_bytes": after, "capacity_bytes": self._capacity,
                           "oversize": nbytes > self._capacity, "priority_overflow": rid == self._priority})
        return True

    def _mark_failed(self, rid: str) -> None:
        with self._lock:
            self._received[rid].append((FAILED_LAYER_NAMES, FAILED_PAYLOAD))

    def _recv_completion_loop(self) -> None:
        while not self._closed:
            with self._rdone_cv:
                while not self._rdone:
                    self._rdone_cv.wait()
                handle, rid, names, payload, row = self._rdone.popleft()
            try:
                row["nccl_s"] = self.plane.wait(handle)
                row["total_s"] = (time.monotonic_ns() - row.pop("_start")) / 1e9
                with self._lock:
                    self._received[rid].append((names, payload))
                self._record_stat(row)
            except Exception as exc:
                log.error("recv completion of %s failed: %s", rid, exc)
                self.release_received(rid, int(row["payload_bytes"]))
                self._mark_failed(rid)

    def _reply(self, ident: bytes, code: bytes, rid: str) -> None:
        if self.faults.drop_ack(rid):
            return
        self.faults.maybe_delay()
        self._sock.send_multipart([ident, code])

    def _listen_loop(self) -> None:
        while not self._closed:
            try:
                ident, raw = self._sock.recv_multipart()[:2]
                msg = msgpack.loads(raw, raw=False)
                cmd = msg["cmd"]
                if cmd == "INIT":
                    self.plane.consumer_connect(msg)
                    self._ready = True
                    continue
                rid = msg["request_id"]
                start = time.monotonic_ns()
                if not self._ready:
                    log.error("%s before INIT", cmd)
                    self._reply(ident, ACK_OOM, rid)
                    self._mark_failed(rid)
                    continue
                if cmd == "PUT":
                    specs = [{"shape": msg["shape"], "dtype": msg["dtype"]}]
                elif cmd == "PUT_BUNDLE":
                    specs = msg["body_specs"] + msg["aux_specs"]
                else:
                    log.error("unknown control message %r", cmd)
                    continue
                nbytes = sum(spec_nbytes(s) for s in specs)
                if not self._reserve(rid, nbytes):
                    self._reply(ident, ACK_RETRY, rid)
                    continue
                try:
                    tensors = [self.plane.alloc(tuple(s["shape"]), getattr(torch, s["dtype"])) for s in specs]
                except (torch.cuda.OutOfMemoryError, RuntimeError) as exc:
                    log.error("allocation for %s failed: %s", rid, exc)
                    self.release_received(rid, nbytes)
                    self._reply(ident, ACK_OOM, rid)
                    self._mark_failed(rid)
                    continue
                self._reply(ident, ACK_OK, rid)
                handle = self.plane.recv(tensors)
                if cmd == "PUT":
                    payload, kind = tensors[0], "raw"
                else:
                    nb = len(msg["body_specs"])
                    payload = {"__bundle__": True, "meta": msg["meta"], "body_chunks": tensors[:nb],
                               "aux_tensors": tensors[nb:]}
                    kind = "bundle"
                row = {"direction": "recv", "kind": kind, "request_id": rid, "payload_bytes": nbytes, "_start": start}
                with self._rdone_cv:
                    self._rdone.append((handle, rid, msg["layer_names"], payload, row))
                    self._rdone_cv.notify()
            except zmq.ZMQError:
                if self._closed:
                    return
                raise
            except Exception as exc:
                log.error("listener error: %s", exc)

    # ------------------------------------------------------------------ stats
    def _record_stat(self, row: dict) -> None:
        if not self._stats_path:
            return
        rec = {"timestamp_ns": time.time_ns(), "pid": os.getpid(), "channel_rank": self.channel_rank, **row}
        try:
            with self._stats_lock, open(self._stats_path, "a", encoding="utf-8") as f:
                f.write(json.dumps(rec, sort_keys=True) + "\n")
        except OSError as exc:
            log.warning("cannot write transport stats to %s: %s", self._stats_path, exc)

    def record_stat(self, row: dict) -> None:
        self._record_stat(row)

    def close(self) -> None:
        self._closed = True
        try:
            self._sock.close(0)
            self._ctx.term()
        except Exception:
            pass
        self.plane.close()
