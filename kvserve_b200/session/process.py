"""Out-of-process session helper (role of
kvsfuse-vllm0.30.0/mooncake/session_ipc.py:25-204 and
session_process.py:1119-1284).

The helper process owns the ZeroMQ sockets, the session state machines,
slot scheduling and timeouts; the engine process keeps only the GPU work.
When a service needs a kernel run it sends a short job over a
``multiprocessing`` pipe and blocks on its result:

* ``EncodeChunkJob`` (producer) -> ``(data_bytes, payload_bytes)``;
* ``DecodeChunkJob`` (consumer) -> ``None``;
* ``DrainSlotsJob`` (either side, at shutdown) -> ``None``.

Control requests from the engine (``AddSend``, ``Open``, ``Abort``,
``Stop``) travel the other way on a second pipe, and ``SessionDone`` reports
ended sessions back.  The session connector runs its service in this helper
with ``KVSERVE_SESSION_PROCESS=1`` (or ``session_process`` in its extra
config); otherwise the same service runs on a thread of the engine process.
Jobs carry everything a GPU job needs that lives in the helper (the
consumer's metadata with its arena handle, the valid token counts after
suffix trimming); objects that cannot cross a pipe (CUDA events) stay in the
engine process, keyed by transfer id.
"""
from __future__ import annotations

import multiprocessing as mp
import os
from dataclasses import dataclass
from typing import Any, Callable, Optional

from .service import ConsumerService, ProducerService


def session_process_enabled() -> bool:
    return os.environ.get("KVSERVE_SESSION_PROCESS", "0").strip().lower() in {"1", "true", "yes", "on"}


# ----------------------------------------------------------------- messages
@dataclass(frozen=True)
class EncodeChunkJob:
    transfer_id: str
    chunk_id: int
    slot_id: int
    slot_offset: int
    flag_index: int
    local_block_ids: Any
    remote_block_ids: Any
    send_meta: Any
    remote_meta: Any = None             # the consumer's XferMetadata (arena handle, slot size)
    valid_tokens_by_group: Any = None


@dataclass(frozen=True)
class DecodeChunkJob:
    transfer_id: str
    d_req_id: str
    chunk_id: int
    slot_id: int
    slot_offset: int
    block_ids: Any
    payload_bytes: int
    valid_tokens_by_group: Any = None


@dataclass(frozen=True)
class DrainSlotsJob:
    reason: str


@dataclass(frozen=True)
class AddSend:
    transfer_id: str
    local_block_ids: Any
    num_tokens: int
    send_meta: Any = None


@dataclass(frozen=True)
class Open:
    endpoint: str
    transfer_id: str
    d_req_id: str
    block_ids: Any
    num_tokens: int
    block_size: int = 16
    logical_blocks_per_chunk: int = 1


@dataclass(frozen=True)
class Abort:
    transfer_id: str
    reason: str


@dataclass(frozen=True)
class Stop:
    pass


@dataclass(frozen=True)
class SessionDone:
    transfer_id: str
    state: str
    error: Optional[str]
    completed_chunks: int
    total_chunks: int = 0


# ------------------------------------------------------------ helper side
def _helper_main(role: str, cfg: dict, ctl, jobs) -> None:
    def run_job(job):
        jobs.send(job)
        ok, value = jobs.recv()
        if not ok:
            raise RuntimeError(value)
        return value

    if role == "producer":
        svc = ProducerService(cfg["endpoint"], lambda s, m: run_job(EncodeChunkJob(
            s.transfer_id, m.chunk_id, m.slot_id, m.slot_offset, m.flag_index, s.local_block_ids,
            s.remote_block_ids, s.send_meta, s.remote_meta, dict(s.valid_tokens_by_group))),
            cfg.get("open_timeout_s", 30.0))
    else:
        def done(s):
            ctl.send(SessionDone(s.transfer_id, s.state.name, s.error, s.completed_chunks, s.total_chunks))
        svc = ConsumerService(cfg["name"], cfg["num_slots"], cfg["slot_bytes"], lambda s, slot, m: run_job(
            DecodeChunkJob(s.transfer_id, s.d_req_id, m.chunk_id, slot.slot_id, slot.offset, s.block_ids,
                           m.payload_bytes, dict(s.valid_tokens_by_group))), done,
            cfg.get("session_timeout_s", 60.0), cfg.get("arena_ipc_handle", b""), cfg.get("flags_ipc_handle", b""))
    ctl.send("ready")
    try:
        while True:
            while ctl.poll(0):
                req = ctl.recv()
                if isinstance(req, Stop):
                    run_job(DrainSlotsJob("stop"))
                    return
                if isinstance(req, AddSend):
                    svc.add_send(req.transfer_id, req.local_block_ids, req.num_tokens, req.send_meta)
                elif isinstance(req, Open):
                    svc.open(req.endpoint, req.transfer_id, req.d_req_id, req.block_ids, req.num_tokens,
                             req.block_size, req.logical_blocks_per_chunk)
                elif isinstance(req, Abort):
                    # a producer withdraws its registered send; a consumer aborts its session
                    (svc.cancel if role == "producer" else svc.abort)(req.transfer_id, req.reason)
            svc.poll(5)
            if role == "producer":
                for s in svc.finished:
                    ctl.send(SessionDone(s.transfer_id, s.state.name, s.error, s.completed_chunks, s.total_chunks))
                svc.finished.clear()
            else:
                svc.finished.clear()
    finally:
        svc.close()


# ------------------------------------------------------------ engine side
class SessionProcess:
    """Engine-side handle of a helper process.  ``handlers`` maps job types
    to callables run in the engine process; :meth:`serve_jobs` must be called
    regularly (e.g. once per engine step) to execute pending jobs."""

    def __init__(self, role: str, cfg: dict, handlers: dict[type, Callable]):
        if role not in ("producer", "consumer"):
            raise ValueError("role must be producer or consumer")
        ctx = mp.get_context("spawn")
        self.ctl, ctl_child = ctx.Pipe()
        self.jobs, jobs_child = ctx.Pipe()
        self.handlers = handlers
        self.done: list[SessionDone] = []
        self.proc = ctx.Process(target=_helper_main, args=(role, cfg, ctl_child, jobs_child), daemon=True,
                                name=f"kvs-session-{role}")
        self.proc.start()
        if not self.ctl.poll(60) or self.ctl.recv() != "ready":
            self.proc.kill()
            raise RuntimeError("session helper did not start")

    def request(self, msg) -> None:
        self.ctl.send(msg)

    def serve_jobs(self, timeout_s: float = 0.0) -> int:
        n = 0
        try:
            while self.jobs.poll(timeout_s if n == 0 else 0):
                job = self.jobs.recv()
                try:
                    result = (True, self.handlers[type(job)](job))
                except Exception as exc:
                    result = (False, f"{type(exc).__name__}: {exc}")
                self.jobs.send(result)
                n += 1
            while self.ctl.poll(0):
                msg = self.ctl.recv()
                if isinstance(msg, SessionDone):
                    self.done.append(msg)
        except (EOFError, BrokenPipeError, ConnectionResetError):
            pass  # the helper has exited
        return n

    def stop(self, timeout_s: float = 10.0) -> None:
        if self.proc.is_alive():
            self.ctl.send(Stop())
            import time
            deadline = time.monotonic() + timeout_s
            while self.proc.is_alive() and time.monotonic() < deadline:
                self.serve_jobs(0.05)
            self.proc.join(1)
            if self.proc.is_alive():
                self.proc.kill()
