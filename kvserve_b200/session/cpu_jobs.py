"""CPU jobs for the session protocol: the same chunked pull as
:mod:`.gpu_jobs`, for peers without a GPU (CPU-only deployments, tests of
the protocol with real compressed frames).

* the consumer's receive arena is a POSIX shared-memory segment
  (:class:`SharedArena`); its name travels in the session metadata where
  the GPU path puts a CUDA IPC handle;
* :class:`CpuEncodeJob` (producer) encodes the pulled chunk with the CPU
  runtime (``create_runtime(device="cpu")``) — K part, then V part — and
  writes each payload into the granted slot of the consumer's segment, the
  way the GPU job's kernels store into the peer's arena;
* :class:`CpuDecodeJob` (consumer) decodes the slot into the session's
  paged blocks.

A consumer on another node exports no segment (``arena=None`` and an empty
handle): the producer's job then returns the slot's bytes, the service sends
them inline in ``ChunkReady``, and the decode job reads them from there.

Payloads in the segment are laid out exactly as on the GPU path (K at the
slot offset, V half a slot further, each part ``part_bytes`` long).
"""
from __future__ import annotations

from multiprocessing import shared_memory

import torch

from .gpu_jobs import _chunk, _valid, part_bytes


class SharedArena:
    """``num_slots`` receive slots of ``slot_bytes`` in one shared-memory
    segment; ``handle`` (its name) goes into the session metadata."""

    def __init__(self, num_slots: int, slot_bytes: int):
        self.slot_bytes = (slot_bytes + 255) // 256 * 256
        self.num_slots = num_slots
        self.shm = shared_memory.SharedMemory(create=True, size=num_slots * self.slot_bytes)
        self.handle = self.shm.name.encode()
        self.view = torch.frombuffer(self.shm.buf, dtype=torch.uint8)

    def close(self) -> None:
        if self.shm is not None:
            del self.view
            self.shm.close()
            self.shm.unlink()
            self.shm = None


class CpuEncodeJob:
    """Producer ``encode_job(session, pull)`` over a bound CPU runtime."""

    def __init__(self, runtime, block_size: int, per_chunk: int):
        self.rt, self.block_size, self.per_chunk = runtime, block_size, per_chunk
        self.part = part_bytes(runtime)
        self._mapped: dict[bytes, tuple] = {}

    def _arena(self, handle: bytes) -> torch.Tensor:
        m = self._mapped.get(handle)
        if m is None:
            shm = shared_memory.SharedMemory(name=handle.decode())
            m = (shm, torch.frombuffer(shm.buf, dtype=torch.uint8))
            self._mapped[handle] = m
        return m[1]

    def __call__(self, session, pull):
        meta = session.remote_meta
        if meta is None:
            raise RuntimeError("no consumer metadata")
        if meta.slot_bytes < 2 * self.part:
            raise RuntimeError(f"consumer slots of {meta.slot_bytes} bytes can not hold 2 x {self.part}")
        # an exported arena is written in place; without one (a consumer on
        # another node) the slot's bytes go back inline in the reply
        arena = self._arena(meta.arena_ipc_handle) if meta.arena_ipc_handle else None
        staged = torch.zeros(2 * self.part, dtype=torch.uint8) if arena is None else None
        blocks = _chunk(session.local_block_ids[0], pull.chunk_id, self.per_chunk)
        valid = _valid(session.valid_tokens_by_group[0], pull.chunk_id, self.per_chunk, self.block_size)
        payload = 0
        for part in (0, 1):
            res = self.rt.encode(0, {0: blocks}, part, valid_tokens_by_group={0: valid})
            n = res.codec_bytes
            if arena is not None:
                off = pull.slot_offset + part * self.part
                arena[off:off + n].copy_(res.payload[:n])
            else:
                staged[part * self.part:part * self.part + n].copy_(res.payload[:n])
            payload += n
        data = 2 * valid * sum(e.heads * e.head_size for e in self.rt.layout.layers) * 2
        if staged is not None:
            return data, payload, staged.numpy().tobytes()
        return data, payload

    def close(self) -> None:
        segments = [shm for shm, _ in self._mapped.values()]
        self._mapped = {}          # drops the tensor views first: a segment with live views can not close
        for shm in segments:
            shm.close()


class CpuDecodeJob:
    """Consumer ``decode_job(session, slot, ready)`` reading its shared arena."""

    def __init__(self, runtime, arena: SharedArena, block_size: int, per_chunk: int):
        self.rt, self.arena, self.block_size, self.per_chunk = runtime, arena, block_size, per_chunk
        self.part = part_bytes(runtime)

    def __call__(self, session, slot, ready) -> None:
        blocks = _chunk(session.block_ids[0], ready.chunk_id, self.per_chunk)
        valid = _valid(session.valid_tokens_by_group[0], ready.chunk_id, self.per_chunk, self.block_size)
        buf = self.rt.receive_buffer(0)
        n = min(self.part, buf.numel())
        inline = getattr(ready, "inline", b"")
        src = torch.frombuffer(bytearray(inline), dtype=torch.uint8) if inline else None
        for part in (0, 1):
            if src is not None:          # the payload came in the reply
                buf[:n].copy_(src[part * self.part:part * self.part + n])
            else:
                off = slot.offset + part * self.part
                buf[:n].copy_(self.arena.view[off:off + n])
            self.rt.decode(0, {0: blocks}, part, codec_bytes=n, valid_tokens_by_group={0: valid})
