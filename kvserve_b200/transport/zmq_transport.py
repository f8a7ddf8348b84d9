"""Host-memory KV transport over ZeroMQ PUSH/PULL (role of
kvserve_v1/transport/zmq_transport.py:20-80, the reference's legacy path).

The consumer binds a PULL socket and a background thread stores arrivals;
the producer connects a PUSH socket.  A message is two frames: a JSON header
``{"request_id", "layer_names", "dtype", "shape"}`` and the tensor's raw
bytes (host copy).  Unlike the reference, the payload is not pickled: the
receiver rebuilds the tensor from dtype + shape, so a peer can never make it
execute code.  Device tensors are staged through host memory; this path is
for tooling and tests, the product hand-off is :mod:`kvserve_b200.transport.p2p`.
"""
from __future__ import annotations

import json
import threading
from typing import Optional

import numpy as np
import torch
import zmq

_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16, "uint8": torch.uint8,
           "int8": torch.int8, "int32": torch.int32, "int64": torch.int64}


class ZmqTransport:
    def __init__(self, is_sender: bool, host: str, port: int, linger_ms: int = 1000):
        self.is_sender = is_sender
        self._ctx = zmq.Context()
        if is_sender:
            self._sock = self._ctx.socket(zmq.PUSH)
            self._sock.setsockopt(zmq.LINGER, linger_ms)
            self._sock.connect(f"tcp://{host}:{port}")
        else:
            self._sock = self._ctx.socket(zmq.PULL)
            self._sock.setsockopt(zmq.RCVTIMEO, 100)
            self._sock.bind(f"tcp://{host}:{port}")
            self._lock = threading.Lock()
            self._received: dict[str, tuple[list[str], torch.Tensor]] = {}
            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._recv_loop, daemon=True, name="kvs-zmq-recv")
            self._thread.start()

    # ------------------------------------------------------------- producer
    def send(self, request_id: str, layer_names: list[str], stacked_kv: torch.Tensor) -> None:
        assert self.is_sender, "send() on a consumer transport"
        t = stacked_kv.detach().contiguous().cpu()
        name = str(t.dtype).replace("torch.", "")
        if name not in _DTYPES:
            raise TypeError(f"unsupported dtype {t.dtype}")
        header = {"request_id": request_id, "layer_names": list(layer_names), "dtype": name,
                  "shape": list(t.shape)}
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        self._sock.send_multipart([json.dumps(header).encode(), raw])

    def wait_for_sent(self) -> None:
        """Sends are handed to ZeroMQ's queue synchronously: nothing to wait for."""
        assert self.is_sender

    # ------------------------------------------------------------- consumer
    def _recv_loop(self) -> None:
        while not self._stop.is_set():
            try:
                head, body = self._sock.recv_multipart()
            except zmq.Again:
                continue
            except zmq.ZMQError:
                break
            h = json.loads(head.decode())
            dtype = _DTYPES[h["dtype"]]
            buf = torch.from_numpy(np.frombuffer(body, dtype=np.uint8).copy()) if body else torch.empty(0, dtype=torch.uint8)
            t = buf.view(dtype).reshape(h["shape"])
            with self._lock:
                self._received[h["request_id"]] = (h["layer_names"], t)

    def drain_received(self) -> dict[str, tuple[list[str], torch.Tensor]]:
        assert not self.is_sender, "drain_received() on a producer transport"
        with self._lock:
            out = dict(self._received)
            self._received.clear()
        return out

    def close(self) -> None:
        if not self.is_sender:
            self._stop.set()
            self._thread.join(timeout=2)
        self._sock.close()
        self._ctx.term()
