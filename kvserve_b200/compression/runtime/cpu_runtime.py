"""The runtime API on the CPU (role of the reference runtime's standard
Python backend and its CPU FWHT path, kvserve_v1/compression/runtime/
pipeline.py:296-335 and 702-720): the same frames, slots, wire profile and
calls as :class:`~kvserve_b200.compression.runtime.manager.CompressionRuntime`,
computed by the frame format's CPU reference encoder and decoder
(:func:`~kvserve_b200.ops.kv_codec.cpu_encode_frame` /
:func:`~kvserve_b200.ops.kv_codec.cpu_decode_frame`) and the lossless
codec's CPU implementation.

It serves peers without a GPU (CPU-only deployments and tests of the layers
above the runtime) and checks the GPU runtime from the outside: both lay the
same frames out in the same slots.  ``create_runtime`` returns it when the
device is the CPU.  Encode and decode run synchronously; the returned
"events" are already complete.
"""
from __future__ import annotations

import threading
from typing import Any, Optional

import numpy as np
import torch

from ...ops import kv_codec as kc
from ..heads import rademacher_signs
from .manager import RUNTIME_SEQ, CompressionRuntime, EncodeResult, _part_index, _Slot
from .memory import CompressionMemoryPlan, frame_spec

RZE_CHUNK = 16384   # the GPU runtime's lossless chunk


class _Done:
    """A completed event (the CPU runtime works synchronously)."""

    def synchronize(self) -> None:
        return

    def query(self) -> bool:
        return True


class CpuCompressionRuntime(CompressionRuntime):
    def __init__(self, plan: CompressionMemoryPlan, kv_cache_layout: str = "HND", blocks_per_logical: int = 1,
                 device=None, execution: str = "both", pipeline_backend: Optional[str] = None):
        if execution not in ("both", "encode", "decode"):
            raise ValueError("Unknown execution capability")
        if kv_cache_layout.upper() not in ("HND", "NHD"):
            raise ValueError("kv_cache_layout must be HND or NHD")
        self.plan, self.config, self.layout = plan, plan.config, plan.layout
        self.execution = execution
        self.hnd = kv_cache_layout.upper() == "HND"
        self.blocks_per_logical = blocks_per_logical
        self.device = torch.device("cpu")
        self.bulk = torch.zeros(self.config.slot_count * plan.slot_bytes, dtype=torch.uint8)
        self.slots = []
        lay = self.layout
        for i in range(self.config.slot_count):
            base = i * plan.slot_bytes
            arena = self.bulk[base: base + lay.arena_bytes]
            off = base + lay.arena_bytes
            out = self.bulk[off: off + lay.codec_capacity] if self.config.uses_codec else None
            self.slots.append(_Slot(arena, out, None, torch.zeros(1, dtype=torch.int64)))
        self.output_slots = []
        self._status = torch.zeros(4, dtype=torch.int32)
        self._bound = False
        self.wire_profile = None
        self._lock = threading.Lock()

    def bind_kv_caches(self, kv_caches: dict, layer_to_group: Optional[dict] = None) -> None:
        super().bind_kv_caches(kv_caches, layer_to_group)
        self._signs = [rademacher_signs(self.config.seed, e.layer_index, e.heads, e.head_size).to(torch.float32)
                       for e in self.layout.layers]

    # ------------------------------------------------------------ helpers
    def _tokens_of(self, cache: torch.Tensor, table: torch.Tensor, T: int) -> torch.Tensor:
        """``[T, H, D]`` of the table's blocks of one layer part."""
        blocks = cache.index_select(0, table.long())
        if self.hnd:                                # [n, H, bs, D] -> [n, bs, H, D]
            blocks = blocks.permute(0, 2, 1, 3)
        return blocks.reshape(-1, blocks.shape[2], blocks.shape[3])[:T]

    def _write_tokens(self, cache: torch.Tensor, table: torch.Tensor, x: torch.Tensor) -> None:
        bs = self.layout.block_size
        for i, blk in enumerate(table.tolist()):
            rows = x[i * bs:(i + 1) * bs]
            if rows.numel() == 0:
                break
            if self.hnd:
                cache[blk, :, :rows.shape[0]] = rows.permute(1, 0, 2).to(cache.dtype)
            else:
                cache[blk, :rows.shape[0]] = rows.to(cache.dtype)

    # ------------------------------------------------------------ encode
    def encode(self, slot_id: int, block_ids_by_group: Any, kv_part: Any,
               valid_tokens_by_group: Any = None, output_slot: Optional[int] = None,
               dest_ptr: Optional[int] = None) -> EncodeResult:
        if not self._bound:
            raise RuntimeError("bind_kv_caches() first")
        if self.execution == "decode":
            raise RuntimeError("this runtime was created for decode only")
        if dest_ptr is not None:
            raise ValueError("the CPU runtime encodes into its own slots (no device address)")
        part = _part_index(kv_part)
        slot = self.slots[slot_id]
        table = self._table(block_ids_by_group)
        T = self._tokens(table, valid_tokens_by_group)
        lay = self.layout
        with slot.lock:
            for e in lay.layers:
                spec = frame_spec(self.config, e, part, T)
                k = self._tokens_of(self._k[e.dense_index], table, T)
                v = self._tokens_of(self._v[e.dense_index], table, T)
                buf = kc.cpu_encode_frame(k, v, spec, self.orders[e.dense_index].cpu(), self._signs[e.dense_index],
                                          layer=e.dense_index, seq=RUNTIME_SEQ)
                base = e.dense_index * lay.frame_stride
                slot.arena[base:base + len(buf)] = torch.frombuffer(buf, dtype=torch.uint8)
            payload, total = slot.arena, None
            if self.config.uses_codec:
                from ..codec.lossless import encode_bytes
                enc = encode_bytes(slot.arena.numpy(), RZE_CHUNK)
                out = slot.codec_out if output_slot is None else self.output_slots[output_slot]
                out[:len(enc)] = torch.frombuffer(bytearray(enc), dtype=torch.uint8)
                slot.codec_total.fill_(len(enc))
                payload, total = out, slot.codec_total
            elif output_slot is not None:
                out = self.output_slots[output_slot]
                out[:lay.arena_bytes].copy_(slot.arena)
                payload = out[:lay.arena_bytes]
            slot.generation += 1
        return EncodeResult(_Done(), payload, lay.arena_bytes, 0, total)

    # ------------------------------------------------------------ decode
    def decode(self, slot_id: int, block_ids_by_group: Any, kv_part: Any, codec_bytes: Optional[int] = None,
               u8_bytes: Optional[int] = None, valid_tokens_by_group: Any = None,
               src_ptr: Optional[int] = None):
        if not self._bound:
            raise RuntimeError("bind_kv_caches() first")
        if self.execution == "encode":
            raise RuntimeError("this runtime was created for encode only")
        if src_ptr is not None:
            raise ValueError("the CPU runtime decodes from its own slots (no device address)")
        part = _part_index(kv_part)
        slot = self.slots[slot_id]
        table = self._table(block_ids_by_group)
        T = self._tokens(table, valid_tokens_by_group)
        lay = self.layout
        with slot.lock:
            frames = slot.arena
            if self.config.uses_codec:
                from ..codec.lossless import decode_bytes
                n = int(codec_bytes) if codec_bytes is not None else slot.codec_out.numel()
                raw = decode_bytes(slot.codec_out[:n].numpy().tobytes())
                frames = torch.from_numpy(np.ascontiguousarray(raw[:lay.arena_bytes]))
            for e in lay.layers:
                spec = frame_spec(self.config, e, part, T)
                base = e.dense_index * lay.frame_stride
                nbytes = kc.frame_layout(spec).frame_bytes
                k, v = kc.cpu_decode_frame(frames[base:base + nbytes].numpy().tobytes(), spec,
                                           self.orders[e.dense_index].cpu(), self._signs[e.dense_index])
                dst = self._k[e.dense_index] if part == 0 else self._v[e.dense_index]
                self._write_tokens(dst, table, k if part == 0 else v)
        return _Done()

    def check_status(self) -> None:
        return

    def shutdown(self) -> None:
        self.slots = []
        self.output_slots = []
        self.bulk = torch.empty(0, dtype=torch.uint8)
