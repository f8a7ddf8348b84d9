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
completion threads retire events in order), ``"ipc"`` (CUDA IPC: the
consumer exports one device receive pool, its ACK names the granted ranges
as a third frame, the producer's copy engine writes them over NVLink — or
within one GPU when both engines share it — and a ``DONE {request_id,
ticket}`` message publishes the payload; no NCCL) or ``"gloo"`` (CPU tensors
over a 2-rank gloo group; used for CPU runs and failure tests).
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


class _RangePool:
    """First-fit allocator of byte ranges in one receive pool (256-byte aligned)."""

    ALIGN = 256

    def __init__(self, size: int):
        self.size = size
        self._free: list[list[int]] = [[0, size]]   # sorted [offset, length]

    def alloc(self, nbytes: int) -> Optional[int]:
        n = max(self.ALIGN, -(-nbytes // self.ALIGN) * self.ALIGN)
        for i, (off, length) in enumerate(self._free):
            if length >= n:
                if length == n:
                    self._free.pop(i)
                else:
                    self._free[i] = [off + n, length - n]
                return off
        return None

    def free(self, off: int, nbytes: int) -> None:
        n = max(self.ALIGN, -(-nbytes // self.ALIGN) * self.ALIGN)
        self._free.append([off, n])
        self._free.sort()
        merged: list[list[int]] = []
        for o, ln in self._free:
            if merged and merged[-1][0] + merged[-1][1] == o:
                merged[-1][1] += ln
            else:
                merged.append([o, ln])
        self._free = merged

    def free_bytes(self) -> int:
        return sum(ln for _, ln in self._free)


class _IpcPlane:
    """CUDA-IPC data plane (see the module docstring).  Consumer: one pool of
    ``capacity`` bytes; a payload that does not fit the pool's free ranges
    (an admitted oversize or priority payload) gets its own allocation,
    exported the same way and freed with the payload's credit."""

    kind = "ipc"

    def __init__(self, device: torch.device, capacity: int = 0, timeout_s: float = 60.0):
        self.device = device
        self.timeout_s = timeout_s
        self.capacity = capacity
        self.stream = None
        self.pool_ptr = 0
        self.pool_handle = b""
        self._pool: Optional[_RangePool] = None
        self._held: dict[str, deque] = defaultdict(deque)   # request -> granted ranges, oldest first
        self._lock = threading.Lock()
        self._tickets: dict[int, threading.Event] = {}
        self._next_ticket = 0
        self._mapped: dict[bytes, int] = {}                  # producer: handle -> mapped base

    # --- consumer
    def producer_init(self) -> dict:
        return {}

    def producer_connect(self) -> None:
        self.stream = torch.cuda.Stream(device=self.device)

    def consumer_connect(self, msg: dict) -> None:
        from ..ops import ext
        if self.pool_ptr:
            return
        with torch.cuda.device(self.device):
            self.pool_ptr = ext().dev_alloc(self.capacity)
            self.pool_handle = ext().ipc_get_handle(self.pool_ptr)
        self._pool = _RangePool(self.capacity)

    def grant(self, rid: str, specs: list) -> tuple[list, dict]:
        """Ranges for ``specs``; returns (tensors, ACK info for the producer)."""
        from ..ops import dtype_code, ext
        tensors, grants, ranges = [], [], []
        with self._lock:
            try:
                for sp in specs:
                    dt = getattr(torch, sp["dtype"])
                    nbytes = max(1, math.prod(sp["shape"]) * torch.tensor([], dtype=dt).element_size())
                    off = self._pool.alloc(nbytes)
                    if off is not None:
                        ptr, grant, rng = self.pool_ptr + off, ["pool", off], ("pool", off, nbytes)
                    else:
                        with torch.cuda.device(self.device):
                            ptr = ext().dev_alloc(nbytes)
                        grant, rng = ["own", ext().ipc_get_handle(ptr)], ("own", ptr, nbytes)
                    ranges.append(rng)
                    tensors.append(ext().tensor_from_ptr(ptr, list(sp["shape"]), dtype_code(dt),
                                                         self.device.index))
                    grants.append(grant)
            except Exception:
                self._free_ranges(ranges)
                raise
            self._held[rid].append(ranges)
            ticket = self._next_ticket
            self._next_ticket += 1
            self._tickets[ticket] = threading.Event()
        return tensors, {"pool": self.pool_handle, "grants": grants, "ticket": ticket}

    def alloc(self, shape, dtype) -> torch.Tensor:
        # the other planes allocate receive tensors here; this one places
        # them inside the exported pool with grant()
        raise RuntimeError("the IPC data plane places received tensors with grant(), not alloc()")

    def recv(self, tensors: list, ticket: int = -1):
        return (time.perf_counter(), self._tickets[ticket], ticket)

    def done(self, ticket: int) -> None:
        ev = self._tickets.get(ticket)
        if ev is not None:
            ev.set()

    def wait(self, handle) -> float:
        t0, ev, ticket = handle
        ok = ev.wait(self.timeout_s)
        with self._lock:
            self._tickets.pop(ticket, None)
        if not ok:
            raise TimeoutError(f"no DONE for ticket {ticket} within {self.timeout_s} s")
        return time.perf_counter() - t0

    def release(self, rid: str) -> None:
        with self._lock:
            q = self._held.get(rid)
            if not q:
                return
            ranges = q.popleft()
            if not q:
                self._held.pop(rid, None)
            self._free_ranges(ranges)

    def _free_ranges(self, ranges: list) -> None:
        from ..ops import ext
        for kind, where, nbytes in ranges:
            if kind == "pool":
                self._pool.free(where, nbytes)
            else:
                with torch.cuda.device(self.device):
                    ext().dev_free(where)

    # --- producer
    def _base(self, handle: bytes) -> int:
        from ..ops import ext
        base = self._mapped.get(handle)
        if base is None:
            with torch.cuda.device(self.device):
                base = ext().ipc_open_handle(handle)
            self._mapped[handle] = base
        return base

    def send(self, tensors: list, ready: Optional[torch.cuda.Event], info: Optional[dict] = None):
        """Copy every tensor into its granted range (copy engine, peer or
        local) and wait for the copies; returns the device seconds."""
        from ..ops import dtype_code, ext
        opened = []
        with torch.cuda.device(self.device), torch.cuda.stream(self.stream):
            if ready is not None:
                self.stream.wait_event(ready)
            start = torch.cuda.Event(enable_timing=True)
            done = torch.cuda.Event(enable_timing=True)
            start.record(self.stream)
            pool = self._base(info["pool"])
            for t, (kind, where) in zip(tensors, info["grants"]):
                if kind == "pool":
                    ptr = pool + int(where)
                else:
                    ptr = ext().ipc_open_handle(where)
                    opened.append(ptr)
                dst = ext().tensor_from_ptr(ptr, list(t.shape), dtype_code(t.dtype), self.device.index)
                dst.copy_(t, non_blocking=True)
            done.record(self.stream)
        done.synchronize()
        with torch.cuda.device(self.device):
            for p in opened:
                ext().ipc_close(p)
        return start.elapsed_time(done) / 1e3

    def close(self) -> None:
        from ..ops import ext
        try:
            with torch.cuda.device(self.device):
                for base in self._mapped.values():
                    ext().ipc_close(base)
                self._mapped.clear()
                for rid in list(self._held):
                    while self._held.get(rid):
                        self.release(rid)
                if self.pool_ptr:
                    ext().dev_free(self.pool_ptr)
                    self.pool_ptr = 0
        except Exception as exc:   # best effort at shutdown
            log.warning("ipc data plane close: %s", exc)


# -------------------------------------------------------------------- transport
class NcclTransport:
    def __init__(self, is_sender: bool, host: str, port: int, local_rank: int = 0, channel_rank: int = 0,
                 recv_buffer_size: int = 1_000_000_000, data_plane: str = "nccl",
                 faults: Optional[FaultInjector] = None, control_timeout_s: float = 60.0):
        self.is_sender = is_sender
        self.local_rank, self.channel_rank = local_rank, channel_rank
        self.port = port + channel_rank
        self.plane_kind = data_plane
        self.device = torch.device(f"cuda:{local_rank}") if data_plane in ("nccl", "ipc") else torch.device("cpu")
        self._stats_path = os.environ.get("KVSERVE_TRANSPORT_STATS_PATH")
        self._stats_lock = threading.Lock()
        self.faults = faults or FaultInjector.from_env()
        self._ctx = zmq.Context()
        self._closed = False
        if data_plane == "nccl":
            self.plane = _NcclPlane(self.device)
        elif data_plane == "gloo":
            self.plane = _GlooPlane(host, port + 1000 + channel_rank)
        elif data_plane == "ipc":
            self.plane = _IpcPlane(self.device, max(1, int(recv_buffer_size)), control_timeout_s)
        else:
            raise ValueError("data_plane must be 'nccl', 'ipc' or 'gloo'")
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
        if self.plane_kind not in ("nccl", "ipc"):
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
        frames = self._sock.recv_multipart()
        ack = frames[0]
        ack_s = time.perf_counter() - t0
        if ack == ACK_RETRY:
            return _RETRY
        if ack != ACK_OK:
            log.error("consumer refused %s (ack=%r)", rid, ack)
            return None
        if self.plane_kind == "ipc":
            info = msgpack.loads(frames[1], raw=False)
            copy_s = self.plane.send(tensors, ready, info)
            self._sock.send(msgpack.dumps({"cmd": "DONE", "request_id": rid, "ticket": info["ticket"]},
                                          use_bin_type=True))
            handle = copy_s
        else:
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
                row["nccl_s"] = float(handle) if self.plane_kind == "ipc" else self.plane.wait(handle)
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
        if self.plane_kind == "ipc":
            self.plane.release(request_id)
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

    def _reply(self, ident: bytes, code: bytes, rid: str, info: Optional[dict] = None) -> None:
        if self.faults.drop_ack(rid):
            return
        self.faults.maybe_delay()
        frames = [ident, code] if info is None else [ident, code, msgpack.dumps(info, use_bin_type=True)]
        self._sock.send_multipart(frames)

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
                if cmd == "DONE":
                    self.plane.done(int(msg["ticket"]))
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
                info = None
                try:
                    if self.plane_kind == "ipc":
                        tensors, info = self.plane.grant(rid, specs)
                    else:
                        tensors = [self.plane.alloc(tuple(s["shape"]), getattr(torch, s["dtype"])) for s in specs]
                except (torch.cuda.OutOfMemoryError, RuntimeError) as exc:
                    log.error("allocation for %s failed: %s", rid, exc)
                    self.release_received(rid, nbytes)
                    self._reply(ident, ACK_OOM, rid)
                    self._mark_failed(rid)
                    continue
                self._reply(ident, ACK_OK, rid, info)
                handle = self.plane.recv(tensors, info["ticket"]) if info is not None else self.plane.recv(tensors)
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
