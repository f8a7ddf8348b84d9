"""Session services: the producer (prefill) and consumer (decode) ends of the
chunked compression session (role of the session state machine in
kvsfuse-vllm0.30.0/mooncake/mooncake_connector.py:1819-2383,3396-3854 and
session_process.py:165-1106).

Both services are single-threaded and poll-driven: the owner calls
:meth:`poll` (from its own loop or from the helper process of
:mod:`.process`).  GPU work is delegated to job callbacks so the services
stay transport- and device-agnostic:

* producer ``encode_job(session, pull) -> (data_bytes, payload_bytes)``:
  encode chunk ``pull.chunk_id`` of ``session`` into the consumer's slot
  (on a node: the fused encode kernel storing through the IPC-mapped
  arena and release-storing flag ``pull.flag_index``); a job that returns
  ``(data_bytes, payload_bytes, payload)`` sends the payload inline in the
  reply instead (a consumer on another node, which exported no arena);
* consumer ``decode_job(session, slot, ready)``: decode the slot into the
  session's paged blocks; ``done_cb(session)`` fires when a session ends.

Messages are two ZeroMQ frames ``[transfer_id, msgpack(message)]`` so an
asynchronous DEALER/ROUTER pair can correlate replies.
"""
from __future__ import annotations

import time
import uuid
from typing import Callable, Optional

import zmq

from .protocol import (ChunkPull, ChunkReady, SessionAbort, SessionAbortAck, SessionOpen, SessionOpened,
                       XferMetadata, decode_request, decode_response, encode_message)
from .state import (ConsumerSession, ProducerSession, ReceiveSlot, ReceiveSlotState, SessionState)
from .tokens import suffix_token_counts


def _chunks(logical_blocks: int, per_chunk: int) -> int:
    return -(-logical_blocks // max(1, per_chunk)) if logical_blocks > 0 else 0


class ProducerService:
    """Prefill side: ROUTER bound on ``endpoint``; answers opens and pulls
    for the transfers registered with :meth:`add_send`.  An open may arrive
    before its send is registered (the consumer's router can be faster than
    the prefill engine's bookkeeping): it waits up to ``open_timeout_s``."""

    def __init__(self, endpoint: str, encode_job: Callable, open_timeout_s: float = 30.0):
        self.ctx = zmq.Context.instance()
        self.sock = self.ctx.socket(zmq.ROUTER)
        self.sock.setsockopt(zmq.LINGER, 0)
        self.sock.bind(endpoint)
        self.encode_job = encode_job
        self.open_timeout_s = open_timeout_s
        self.sessions: dict[str, ProducerSession] = {}
        self.finished: list[ProducerSession] = []
        # opens that arrived before their send was registered: answered by
        # add_send, or refused when the open timeout passes
        self._early: dict[str, tuple[bytes, SessionOpen, float]] = {}
        self.stats = {"opens": 0, "pulls": 0, "aborts": 0, "expired": 0, "payload_bytes": 0, "data_bytes": 0}

    def add_send(self, transfer_id: str, local_block_ids: list, num_tokens: int, send_meta=None) -> None:
        s = ProducerSession(transfer_id, "", local_block_ids=local_block_ids, send_meta=send_meta)
        s.valid_tokens_by_group = {0: num_tokens}
        s.deadline = time.monotonic() + self.open_timeout_s
        self.sessions[transfer_id] = s
        early = self._early.pop(transfer_id, None)
        if early is not None:
            self._on_open(early[0], transfer_id, early[1])

    def _reply(self, ident: bytes, tid: str, msg) -> None:
        self.sock.send_multipart([ident, tid.encode(), encode_message(msg)])

    def _finish(self, s: ProducerSession, state: SessionState) -> None:
        s.move(state)
        self.sessions.pop(s.transfer_id, None)
        self.finished.append(s)

    def _on_open(self, ident: bytes, tid: str, m: SessionOpen) -> None:
        self.stats["opens"] += 1
        s = self.sessions.get(tid)
        meta: XferMetadata = m.metadata
        if s is None and tid in meta.req_blocks:
            self._early[tid] = (ident, m, time.monotonic() + self.open_timeout_s)
            return
        if s is None or s.state is not SessionState.PLANNED or tid not in meta.req_blocks:
            self._reply(ident, tid, SessionOpened(0, 0, error=f"unknown or busy transfer {tid}"))
            return
        d_req, remote_blocks = meta.req_blocks[tid]
        local = s.local_block_ids
        if remote_blocks and local and len(remote_blocks[0]) > len(local[0]):
            self._reply(ident, tid, SessionOpened(0, 0, error=f"{tid}: consumer asks for more blocks than sent"))
            return
        if remote_blocks and local and len(remote_blocks[0]) < len(local[0]):
            # the consumer holds a block-aligned prefix: send the last blocks,
            # counting tokens from the suffix start
            total = s.valid_tokens_by_group[0]
            s.local_block_ids = [ids[len(ids) - len(r):] for ids, r in zip(local, remote_blocks)]
            s.valid_tokens_by_group = suffix_token_counts(total, remote_blocks, {0: meta.block_size})
        s.d_req_id, s.remote_block_ids, s.nonce = d_req, remote_blocks, m.nonce
        s.remote_meta = meta
        s.remote_session = ident.hex()
        s.logical_block_count = len(remote_blocks[0]) if remote_blocks else 0
        s.total_chunks = _chunks(s.logical_block_count, meta.logical_blocks_per_chunk)
        s.move(SessionState.ACTIVE)
        self._reply(ident, tid, SessionOpened(s.logical_block_count, s.total_chunks))
        if s.total_chunks == 0:
            self._finish(s, SessionState.COMPLETE)

    def _on_pull(self, ident: bytes, tid: str, m: ChunkPull) -> None:
        self.stats["pulls"] += 1
        s = self.sessions.get(tid)
        if s is None or s.state is not SessionState.ACTIVE or m.nonce != s.nonce:
            self._reply(ident, tid, ChunkReady(m.chunk_id, 0, 0, error="no active session"))
            return
        s.inflight_chunks += 1
        inline = b""
        try:
            res = self.encode_job(s, m)
            data_bytes, payload_bytes = res[0], res[1]
            if len(res) > 2:             # no arena to write: the payload rides in the reply
                inline = bytes(res[2])
        except Exception as exc:  # the job's failure ends the session, never the service
            s.inflight_chunks -= 1
            s.error = f"encode failed: {exc}"
            self._reply(ident, tid, ChunkReady(m.chunk_id, 0, 0, error=s.error))
            self._finish(s, SessionState.FAILED)
            return
        s.inflight_chunks -= 1
        s.completed_chunks += 1
        self.stats["payload_bytes"] += int(payload_bytes)
        self.stats["data_bytes"] += int(data_bytes)
        self._reply(ident, tid, ChunkReady(m.chunk_id, int(data_bytes), int(payload_bytes), inline=inline))
        if s.completed_chunks >= s.total_chunks:
            self._finish(s, SessionState.COMPLETE)

    def _on_abort(self, ident: bytes, tid: str, m: SessionAbort) -> None:
        self.stats["aborts"] += 1
        self._early.pop(tid, None)
        s = self.sessions.get(tid)
        if s is not None and not s.done:
            s.error = m.reason
            self._finish(s, SessionState.CANCELLED)
        self._reply(ident, tid, SessionAbortAck(tid, m.d_req_id, m.nonce))

    def cancel(self, transfer_id: str, reason: str) -> None:
        """Withdraw a registered send (its blocks are being freed); a later
        open or pull of it is refused."""
        s = self.sessions.get(transfer_id)
        if s is not None and not s.done:
            s.error = reason
            self._finish(s, SessionState.CANCELLED)

    def sweep(self, now: Optional[float] = None) -> list:
        """Expire registered sends that no consumer opened in time."""
        now = time.monotonic() if now is None else now
        out = []
        for tid, (ident, _, deadline) in list(self._early.items()):
            if now > deadline:
                del self._early[tid]
                self._reply(ident, tid, SessionOpened(0, 0, error=f"unknown transfer {tid}"))
        for s in list(self.sessions.values()):
            if s.state is SessionState.PLANNED and now > s.deadline:
                s.error = "open timeout"
                self._finish(s, SessionState.CANCELLED)
                self.stats["expired"] += 1
                out.append(s)
        return out

    def poll(self, timeout_ms: int = 0) -> int:
        n = 0
        while self.sock.poll(timeout_ms if n == 0 else 0):
            ident, tid, body = self.sock.recv_multipart()
            m = decode_request(body)
            t = tid.decode()
            if isinstance(m, SessionOpen):
                self._on_open(ident, t, m)
            elif isinstance(m, ChunkPull):
                self._on_pull(ident, t, m)
            else:
                self._on_abort(ident, t, m)
            n += 1
        self.sweep()
        return n

    def close(self) -> None:
        self.sock.close()


class ConsumerService:
    """Decode side: grants receive slots of its arena and pulls chunks."""

    def __init__(self, name: str, num_slots: int, slot_bytes: int, decode_job: Callable,
                 done_cb: Optional[Callable] = None, session_timeout_s: float = 60.0,
                 arena_ipc_handle: bytes = b"", flags_ipc_handle: bytes = b""):
        self.ctx = zmq.Context.instance()
        self.name = name
        self.slots = [ReceiveSlot(i, i * slot_bytes) for i in range(num_slots)]
        self.slot_bytes = slot_bytes
        self.decode_job, self.done_cb = decode_job, done_cb
        self.session_timeout_s = session_timeout_s
        self.arena_ipc_handle, self.flags_ipc_handle = arena_ipc_handle, flags_ipc_handle
        self.socks: dict[str, zmq.Socket] = {}
        self.sessions: dict[str, ConsumerSession] = {}
        self.endpoint_of: dict[str, str] = {}
        self.finished: list[ConsumerSession] = []
        self.stats = {"chunks": 0, "payload_bytes": 0, "data_bytes": 0, "failed": 0}

    def _sock(self, endpoint: str) -> zmq.Socket:
        s = self.socks.get(endpoint)
        if s is None:
            s = self.ctx.socket(zmq.DEALER)
            s.setsockopt(zmq.LINGER, 0)
            s.setsockopt(zmq.IDENTITY, f"{self.name}-{uuid.uuid4().hex[:8]}".encode())
            s.connect(endpoint)
            self.socks[endpoint] = s
        return s

    def _send(self, tid: str, msg) -> None:
        self._sock(self.endpoint_of[tid]).send_multipart([tid.encode(), encode_message(msg)])

    def open(self, endpoint: str, transfer_id: str, d_req_id: str, block_ids: list, num_tokens: int,
             block_size: int = 16, logical_blocks_per_chunk: int = 1) -> ConsumerSession:
        s = ConsumerSession(transfer_id, d_req_id, block_ids=block_ids, nonce=uuid.uuid4().hex)
        s.valid_tokens_by_group = {0: num_tokens}
        s.deadline = time.monotonic() + self.session_timeout_s
        s.move(SessionState.OPENING)
        self.sessions[transfer_id] = s
        self.endpoint_of[transfer_id] = endpoint
        meta = XferMetadata(self.name, 0, 1, 0, {transfer_id: (d_req_id, block_ids)},
                            arena_ipc_handle=self.arena_ipc_handle, flags_ipc_handle=self.flags_ipc_handle,
                            arena_bytes=self.slot_bytes * len(self.slots), slot_bytes=self.slot_bytes,
                            num_slots=len(self.slots), block_size=block_size, num_tokens=num_tokens,
                            logical_blocks_per_chunk=logical_blocks_per_chunk)
        self._send(transfer_id, SessionOpen(meta, s.nonce))
        return s

    def abort(self, transfer_id: str, reason: str) -> None:
        s = self.sessions.get(transfer_id)
        if s is not None and not s.done:
            self._send(transfer_id, SessionAbort(transfer_id, s.d_req_id, reason, s.nonce))
            self._end(s, SessionState.CANCELLED, reason)

    def _end(self, s: ConsumerSession, state: SessionState, error: Optional[str] = None) -> None:
        for slot in self.slots:
            if slot.owner == s.transfer_id:
                slot.state, slot.chunk_id, slot.owner = ReceiveSlotState.FREE, None, None
        s.error = error or s.error
        s.move(state)
        self.sessions.pop(s.transfer_id, None)
        self.finished.append(s)
        if state is SessionState.FAILED:
            self.stats["failed"] += 1
        if self.done_cb is not None:
            self.done_cb(s)

    def _grant(self) -> None:
        """Hand free slots to active sessions, oldest session first."""
        for s in list(self.sessions.values()):
            if s.state is not SessionState.ACTIVE:
                continue
            while s.next_chunk < s.total_chunks:
                slot = next((x for x in self.slots if x.state is ReceiveSlotState.FREE), None)
                if slot is None:
                    return
                slot.move(ReceiveSlotState.GRANTED, chunk_id=s.next_chunk, owner=s.transfer_id)
                self._send(s.transfer_id, ChunkPull(s.transfer_id, s.d_req_id, s.next_chunk, slot.slot_id,
                                                    slot.offset, slot.slot_id, s.nonce))
                s.next_chunk += 1

    def _on_opened(self, s: ConsumerSession, m: SessionOpened) -> None:
        if m.error:
            self._end(s, SessionState.FAILED, m.error)
            return
        s.logical_block_count, s.total_chunks = m.logical_block_count, m.total_chunks
        s.move(SessionState.ACTIVE)
        if s.total_chunks == 0:
            self._end(s, SessionState.COMPLETE)

    def _on_ready(self, s: ConsumerSession, m: ChunkReady) -> None:
        slot = next((x for x in self.slots if x.owner == s.transfer_id and x.chunk_id == m.chunk_id), None)
        if m.error or slot is None:
            self._end(s, SessionState.FAILED, m.error or f"chunk {m.chunk_id} has no granted slot")
            return
        slot.move(ReceiveSlotState.RECEIVED)
        slot.move(ReceiveSlotState.DECODING)
        try:
            self.decode_job(s, slot, m)
        except Exception as exc:
            self._end(s, SessionState.FAILED, f"decode failed: {exc}")
            return
        slot.move(ReceiveSlotState.WRITEBACK)
        slot.move(ReceiveSlotState.FREE)
        s.completed_chunks += 1
        self.stats["chunks"] += 1
        self.stats["payload_bytes"] += m.payload_bytes
        self.stats["data_bytes"] += m.data_bytes
        if s.completed_chunks >= s.total_chunks:
            s.move(SessionState.DRAINING)
            self._end(s, SessionState.COMPLETE)

    def sweep(self, now: Optional[float] = None) -> None:
        now = time.monotonic() if now is None else now
        for s in list(self.sessions.values()):
            if now > s.deadline:
                self.abort(s.transfer_id, "session timeout")

    def poll(self, timeout_ms: int = 0) -> int:
        n = 0
        socks = list(self.socks.values())
        if not socks and timeout_ms > 0:
            time.sleep(timeout_ms / 1000.0)   # nothing to wait on yet: do not spin
        if socks:
            poller = zmq.Poller()
            for sk in socks:
                poller.register(sk, zmq.POLLIN)
            for sk, _ in poller.poll(timeout_ms):
                while sk.poll(0):
                    tid, body = sk.recv_multipart()
                    m = decode_response(body)
                    s = self.sessions.get(tid.decode())
                    n += 1
                    if s is None:
                        continue  # late reply for a finished session
                    if isinstance(m, SessionOpened):
                        self._on_opened(s, m)
                    elif isinstance(m, ChunkReady):
                        self._on_ready(s, m)
        self._grant()
        self.sweep()
        return n

    def close(self) -> None:
        for s in self.socks.values():
            s.close()
