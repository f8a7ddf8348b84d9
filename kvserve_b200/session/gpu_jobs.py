"""GPU jobs that put the session protocol on the device data path.

:class:`ProducerService` and :class:`ConsumerService` only move control
messages; these callables are their ``encode_job`` / ``decode_job``:

* the consumer exports its receive arena (plain ``cudaMalloc`` memory,
  :class:`ReceiveArena`) through CUDA IPC in the session's metadata, and
  grants slots of it chunk by chunk;
* :class:`RuntimeEncodeJob` (prefill GPU) maps the consumer's arena on
  first use and runs the compression runtime's fused encode of the pulled
  chunk — K frames, then V frames half a slot further — with the output
  pointer IN the consumer's slot: the kernels store over NVLink (or locally
  when both ends share a GPU), and the job synchronises its stream before the
  service replies ChunkReady;
* :class:`RuntimeDecodeJob` (decode GPU) decodes the slot straight into the
  session's paged blocks with the fused decode kernels.

Between nodes (no CUDA IPC), the consumer exports no arena: the encode job
then encodes into its runtime's own slot and returns the bytes, the service
sends them inline in ``ChunkReady``, and the decode job stages them in its
runtime's receive buffer before decoding.

This is the transfer the reference's Mooncake connector performs with its
RDMA engine and session helper process
(kvsfuse-vllm0.30.0/mooncake/mooncake_connector.py:2201-2232, 2251-2383,
3396-3808); here the "RDMA write" is the encode kernel's own peer stores.
"""
from __future__ import annotations

from typing import Optional

import torch

from ..ops import ext


def part_bytes(runtime) -> int:
    """Bytes of one K (or V) part of a chunk in a slot (256-byte aligned)."""
    lay = runtime.layout
    n = lay.codec_capacity if runtime.config.uses_codec else lay.arena_bytes
    return (n + 255) // 256 * 256


class ReceiveArena:
    """``num_slots`` receive slots of ``slot_bytes`` in cudaMalloc memory
    (exportable through CUDA IPC)."""

    def __init__(self, num_slots: int, slot_bytes: int, device=None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.slot_bytes = (slot_bytes + 255) // 256 * 256
        self.num_slots = num_slots
        with torch.cuda.device(self.device):
            self.base = ext().dev_alloc(num_slots * self.slot_bytes)
        self.handle = ext().ipc_get_handle(self.base)

    def close(self) -> None:
        if self.base:
            with torch.cuda.device(self.device):
                ext().dev_free(self.base)
            self.base = 0


def _chunk(ids: list, chunk_id: int, per_chunk: int) -> list:
    return ids[chunk_id * per_chunk:(chunk_id + 1) * per_chunk]


def _valid(total_tokens: int, chunk_id: int, per_chunk: int, block_size: int) -> int:
    return max(0, min(per_chunk * block_size, total_tokens - chunk_id * per_chunk * block_size))


class RuntimeEncodeJob:
    """Producer ``encode_job(session, pull)`` over a bound encode runtime."""

    def __init__(self, runtime, block_size: int, per_chunk: int):
        self.rt, self.block_size, self.per_chunk = runtime, block_size, per_chunk
        self.part = part_bytes(runtime)
        self._mapped: dict[bytes, int] = {}

    def _arena(self, handle: bytes) -> int:
        base = self._mapped.get(handle)
        if base is None:
            with torch.cuda.device(self.rt.device):
                base = ext().ipc_open_handle(handle)
            self._mapped[handle] = base
        return base

    def __call__(self, session, pull):
        meta = session.remote_meta
        if meta is None:
            raise RuntimeError("no consumer metadata")
        if meta.slot_bytes < 2 * self.part:
            raise RuntimeError(f"consumer slots of {meta.slot_bytes} bytes can not hold 2 x {self.part}")
        ready = session.send_meta
        if isinstance(ready, torch.cuda.Event):
            ready.synchronize()    # the forward that wrote these blocks has finished
        blocks = _chunk(session.local_block_ids[0], pull.chunk_id, self.per_chunk)
        valid = _valid(session.valid_tokens_by_group[0], pull.chunk_id, self.per_chunk, self.block_size)
        data = 2 * valid * sum(e.heads * e.head_size for e in self.rt.layout.layers) * 2
        payload = 0
        if not meta.arena_ipc_handle:
            # a consumer on another node: encode into this runtime's slot and
            # return the bytes, which the service sends inline in its reply
            staged = bytearray(2 * self.part)
            for part in (0, 1):
                res = self.rt.encode(0, {0: blocks}, part, valid_tokens_by_group={0: valid})
                res.event.synchronize()
                n = res.codec_bytes
                staged[part * self.part:part * self.part + n] = res.payload[:n].cpu().numpy().tobytes()
                payload += n
            return data, payload, bytes(staged)
        dest = self._arena(meta.arena_ipc_handle) + pull.slot_offset
        for part in (0, 1):
            res = self.rt.encode(0, {0: blocks}, part, valid_tokens_by_group={0: valid},
                                 dest_ptr=dest + part * self.part)
            res.event.synchronize()
            payload += res.codec_bytes
        return data, payload

    def close(self) -> None:
        with torch.cuda.device(self.rt.device):
            for base in self._mapped.values():
                ext().ipc_close(base)
        self._mapped = {}


class RuntimeDecodeJob:
    """Consumer ``decode_job(session, slot, ready)`` over a bound decode
    runtime reading the arena it exported."""

    def __init__(self, runtime, arena: ReceiveArena, block_size: int, per_chunk: int):
        self.rt, self.arena, self.block_size, self.per_chunk = runtime, arena, block_size, per_chunk
        self.part = part_bytes(runtime)

    def __call__(self, session, slot, ready) -> None:
        blocks = _chunk(session.block_ids[0], ready.chunk_id, self.per_chunk)
        valid = _valid(session.valid_tokens_by_group[0], ready.chunk_id, self.per_chunk, self.block_size)
        inline = getattr(ready, "inline", b"")
        if inline:
            # the payload came in the reply: stage it in the runtime's own
            # receive buffer and decode from there
            buf = self.rt.receive_buffer(0)
            n = min(self.part, buf.numel())
            host = torch.frombuffer(bytearray(inline), dtype=torch.uint8)
            for part in (0, 1):
                buf[:n].copy_(host[part * self.part:part * self.part + n])
                self.rt.decode(0, {0: blocks}, part, codec_bytes=n, valid_tokens_by_group={0: valid}).synchronize()
            self.rt.check_status()
            return
        src = self.arena.base + slot.offset
        for part in (0, 1):
            ev = self.rt.decode(0, {0: blocks}, part, codec_bytes=self.part, valid_tokens_by_group={0: valid},
                                src_ptr=src + part * self.part)
            ev.synchronize()
        self.rt.check_status()
