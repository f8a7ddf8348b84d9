"""The fixed-profile compression runtime (API v1; the surface of
kvserve_v1/compression/runtime/manager.py:66-494 and fused_runtime.py),
backed by the sm_100a frame kernels.

* ``bind_kv_caches`` records the caller's per-layer paged K/V tensors
  (``HND`` ``[num_blocks, H, block_size, D]`` or ``NHD`` ``[num_blocks,
  block_size, H, D]``; one ``[2, ...]`` tensor or a ``(K, V)`` pair per layer),
  uploads head orders / sign bits and fixes the ``wire_profile``.
* ``encode(slot, block_ids_by_group, part)`` runs one fused gather + sign +
  FWHT + quantise + pack launch per layer straight from the paged cache into
  the slot's frame arena (no intermediate gather buffer), then the lossless
  stage when the pipeline has a codec.  It returns a CUDA event and the sizes.
* ``decode`` mirrors it: lossless decode, then ONE fused launch over all layers
  writing the destination blocks through a per-layer pointer table.

The runtime owns one bulk allocation carved into slots; it never touches the
network.  Callers fence the returned events before reading payloads, reusing
a slot, or publishing the destination cache.
"""
from __future__ import annotations

import hashlib
import json
import threading
from dataclasses import asdict, dataclass, field
from typing import Any, Optional

import torch

from ... import ops
from ...ops import kv_codec as kc
from ..heads import pack_sign_bits, rademacher_signs
from .config import CompressionConfig
from .memory import ALIGNMENT, CompressionMemoryPlan, frame_spec
from .spec import round_up

WIRE_PREFIX = "kvs-b200-frame-v1:"
RUNTIME_SEQ = 1


@dataclass
class EncodeResult:
    event: torch.cuda.Event
    payload: Optional[torch.Tensor]  # bytes to transfer (frames or codec output), device view; None: written to dest_ptr
    u8_bytes: int                  # frame-arena bytes (what decode expects after the codec)
    raw_tail_bytes: int = 0        # frames carry partial blocks; no separate raw tail
    _codec_bytes: Optional[torch.Tensor] = None

    @property
    def codec_bytes(self) -> int:
        if self._codec_bytes is None:
            return self.u8_bytes
        self.event.synchronize()
        return int(self._codec_bytes.item())


@dataclass
class _Slot:
    arena: torch.Tensor
    codec_out: Optional[torch.Tensor]
    codec_scratch: Optional[torch.Tensor]
    codec_total: torch.Tensor
    lock: threading.Lock = field(default_factory=threading.Lock)
    generation: int = 0


def _part_index(kv_part: Any) -> int:
    if kv_part in (0, "k", "key", "K"):
        return 0
    if kv_part in (1, "v", "value", "V"):
        return 1
    raise ValueError(f"kv_part must be 0/'key' or 1/'value', got {kv_part!r}")


class CompressionRuntime:
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
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.stream = torch.cuda.Stream(self.device, priority=-1)
        self.bulk = torch.empty(self.config.slot_count * plan.slot_bytes, dtype=torch.uint8, device=self.device)
        self.slots: list[_Slot] = []
        lay = self.layout
        for i in range(self.config.slot_count):
            base = i * plan.slot_bytes
            arena = self.bulk[base: base + lay.arena_bytes]
            off = base + lay.arena_bytes
            out = self.bulk[off: off + lay.codec_capacity] if self.config.uses_codec else None
            off += lay.codec_capacity
            scr = self.bulk[off: off + lay.codec_scratch] if self.config.uses_codec else None
            self.slots.append(_Slot(arena, out, scr, torch.zeros(1, dtype=torch.int64, device=self.device)))
        self.output_slots: list[torch.Tensor] = []
        self._enc_state = kc.EncoderState(self.device)
        self._status = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._bound = False
        self.wire_profile: Optional[str] = None

    # ------------------------------------------------------------- binding
    def bind_kv_caches(self, kv_caches: dict, layer_to_group: Optional[dict] = None) -> None:
        lay = self.layout
        self._k, self._v = [], []
        for e in lay.layers:
            t = kv_caches[e.name]
            if isinstance(t, (tuple, list)):
                k, v = t
            elif t.dim() == 5 and t.shape[0] == 2:
                k, v = t[0], t[1]
            else:
                raise ValueError(f"cache of {e.name} must be [2, ...] or a (K, V) pair")
            hd = 1 if self.hnd else 2
            if k.dim() != 4 or k.shape[hd] != e.heads or k.shape[3] != e.head_size or k.dtype != torch.bfloat16:
                raise ValueError(f"cache of {e.name} has shape {tuple(k.shape)}; expected "
                                 f"{'[nb, H, bs, D]' if self.hnd else '[nb, bs, H, D]'} bf16")
            if k.stride() != v.stride():
                raise ValueError("K and V views of a layer must share strides")
            self._k.append(k)
            self._v.append(v)
        sel = self.plan.selection
        orders = torch.tensor([list(sel.local_orders.get(e.layer_index, tuple(range(e.heads)))) for e in lay.layers],
                              dtype=torch.int32)
        signs = torch.stack([rademacher_signs(self.config.seed, e.layer_index, e.heads, e.head_size)
                             for e in lay.layers])
        self.orders = orders.to(self.device)
        self.sign_bits = pack_sign_bits(signs).to(self.device)
        self.n_lows = torch.tensor([e.n_low for e in lay.layers], dtype=torch.int32, device=self.device)
        self.layer_ptrs = torch.tensor([[k.data_ptr(), v.data_ptr()] for k, v in zip(self._k, self._v)],
                                       dtype=torch.int64, device=self.device)
        cfg = {k: v for k, v in asdict(self.config).items() if k not in ("score_path", "slot_count")}
        cfg["pipeline"] = list(cfg["pipeline"])
        ident = {"version": 1, "config": cfg, "layers": [[e.layer_index, e.heads, e.head_size, e.n_low]
                                                        for e in lay.layers],
                 "chunk_tokens": lay.chunk_tokens, "frame_stride": lay.frame_stride, "orders": orders.tolist()}
        self.wire_profile = WIRE_PREFIX + hashlib.sha256(json.dumps(ident, sort_keys=True).encode()).hexdigest()
        self._bound = True

    # ------------------------------------------------------------- sizes
    def data_bytes(self, valid_tokens: Optional[int] = None) -> int:
        return self.layout.arena_bytes

    def aux_bytes(self, *args, **kwargs) -> int:
        return 0  # parameters travel inside each frame

    def registered_memory(self) -> tuple[list[int], list[int]]:
        addrs = [self.bulk.data_ptr()] + [t.data_ptr() for t in self.output_slots]
        lens = [self.bulk.numel()] + [t.numel() for t in self.output_slots]
        return addrs, lens

    def allocate_output_slots(self, n: int) -> list[torch.Tensor]:
        if not 0 <= n <= 16:
            raise ValueError("output slot count must be in [0, 16]")
        if self.output_slots:
            raise RuntimeError("output slots were already allocated")
        cap = self.layout.codec_capacity if self.config.uses_codec else self.layout.arena_bytes
        self.output_slots = [torch.empty(cap, dtype=torch.uint8, device=self.device) for _ in range(n)]
        return self.output_slots

    # ------------------------------------------------------------ helpers
    def _table(self, block_ids_by_group: Any) -> torch.Tensor:
        ids = block_ids_by_group
        if isinstance(ids, dict):
            ids = ids.get(0, next(iter(ids.values())))
        elif isinstance(ids, (list, tuple)) and ids and isinstance(ids[0], (list, tuple, torch.Tensor)):
            ids = ids[0]
        t = torch.as_tensor(ids, dtype=torch.int32)
        if t.numel() * self.layout.block_size > self.layout.chunk_tokens:
            raise ValueError("more blocks than one chunk holds")
        return t.to(self.device, non_blocking=True)

    def _tokens(self, table: torch.Tensor, valid: Any) -> int:
        if valid is None:
            return int(table.numel()) * self.layout.block_size
        if isinstance(valid, dict):
            valid = valid.get(0, next(iter(valid.values())))
        if isinstance(valid, (list, tuple)):
            valid = valid[0]
        return int(valid)

    # ------------------------------------------------------------ encode
    def encode(self, slot_id: int, block_ids_by_group: Any, kv_part: Any,
               valid_tokens_by_group: Any = None, output_slot: Optional[int] = None,
               dest_ptr: Optional[int] = None) -> EncodeResult:
        """Encode one chunk's ``kv_part`` into slot ``slot_id``.  With
        ``dest_ptr`` (a 256-byte aligned device address, local or a peer
        GPU's memory mapped through CUDA IPC) the payload is written there
        instead — the frames directly, or the codec output when the pipeline
        has a codec — so a zero-copy transport needs no staging copy."""
        if not self._bound:
            raise RuntimeError("bind_kv_caches() first")
        if self.execution == "decode":
            raise RuntimeError("this runtime was created for decode only")
        part = _part_index(kv_part)
        slot = self.slots[slot_id]
        table = self._table(block_ids_by_group)
        T = self._tokens(table, valid_tokens_by_group)
        lay = self.layout
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        if dest_ptr is not None and dest_ptr % 256:
            raise ValueError("dest_ptr must be 256-byte aligned")
        with torch.cuda.stream(self.stream):
            direct = dest_ptr is not None and not self.config.uses_codec
            base = dest_ptr if direct else slot.arena.data_ptr()
            for e in lay.layers:
                spec = frame_spec(self.config, e, part, T)
                k, v = self._k[e.dense_index], self._v[e.dense_index]
                kc.encode_layer(k, v, spec, self.orders[e.dense_index], self.sign_bits[e.dense_index],
                                base + e.dense_index * lay.frame_stride, self._enc_state, seq=RUNTIME_SEQ,
                                layer=e.dense_index, part_mask=1 << part, block_table=table, hnd=self.hnd)
            payload, total = (None if direct else slot.arena), None
            if self.config.uses_codec:
                if dest_ptr is not None:
                    out = ops.ext().tensor_from_ptr(int(dest_ptr), [lay.codec_capacity], ops.dtype_code(torch.uint8),
                                                    self.device.index)
                else:
                    out = slot.codec_out if output_slot is None else self.output_slots[output_slot]
                ops.count_launches(3)
                ops.ext().rze_encode(slot.arena, out, slot.codec_scratch, slot.codec_total, 16384)
                payload, total = out, slot.codec_total
            elif output_slot is not None and not direct:
                out = self.output_slots[output_slot]
                out[: lay.arena_bytes].copy_(slot.arena)
                payload = out[: lay.arena_bytes]
            ev = torch.cuda.Event()
            ev.record(self.stream)
        slot.generation += 1
        return EncodeResult(ev, payload, lay.arena_bytes, 0, total)

    def encode_into(self, output_slot: int, slot_id: int, block_ids_by_group: Any, kv_part: Any,
                    valid_tokens_by_group: Any = None) -> EncodeResult:
        return self.encode(slot_id, block_ids_by_group, kv_part, valid_tokens_by_group, output_slot=output_slot)

    def receive_buffer(self, slot_id: int) -> torch.Tensor:
        """Where the transport must land the peer's payload for ``slot_id``."""
        s = self.slots[slot_id]
        return s.codec_out if self.config.uses_codec else s.arena

    # ------------------------------------------------------------ decode
    def decode(self, slot_id: int, block_ids_by_group: Any, kv_part: Any, codec_bytes: Optional[int] = None,
               u8_bytes: Optional[int] = None, valid_tokens_by_group: Any = None,
               src_ptr: Optional[int] = None) -> torch.cuda.Event:
        """Decode slot ``slot_id`` (or the payload at device address
        ``src_ptr``, where a zero-copy transport landed it) into the blocks."""
        if not self._bound:
            raise RuntimeError("bind_kv_caches() first")
        if self.execution == "encode":
            raise RuntimeError("this runtime was created for encode only")
        part = _part_index(kv_part)
        slot = self.slots[slot_id]
        table = self._table(block_ids_by_group)
        T = self._tokens(table, valid_tokens_by_group)
        lay = self.layout
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        with torch.cuda.stream(self.stream):
            frames = slot.arena.data_ptr()
            if self.config.uses_codec:
                src = slot.codec_out if src_ptr is None else ops.ext().tensor_from_ptr(
                    int(src_ptr), [lay.codec_capacity], ops.dtype_code(torch.uint8), self.device.index)
                n = int(codec_bytes) if codec_bytes is not None else src.numel()
                ops.count_launches(2)
                ops.ext().rze_decode(src[:n], slot.arena, slot.codec_scratch, 16384)
            elif src_ptr is not None:
                if src_ptr % 256:
                    raise ValueError("src_ptr must be 256-byte aligned")
                frames = int(src_ptr)
            big = max(lay.layers, key=lambda e: kc.frame_layout(frame_spec(self.config, e, part, T)).frame_bytes)
            spec = frame_spec(self.config, big, part, T)
            template = self._k[0] if part == 0 else self._v[0]
            kc.decode_layers(frames, lay.frame_stride, spec, self.orders, self.sign_bits, template,
                             table, self._status, seq=RUNTIME_SEQ, layer_begin=0, num_layers=len(lay.layers),
                             n_lows=self.n_lows, part_mask=1 << part, layer_ptrs=self.layer_ptrs, hnd=self.hnd)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        return ev

    def check_status(self) -> None:
        code = int(self._status[0].item())
        if code:
            self._status.zero_()
            raise RuntimeError(f"runtime decode failed: {ops.STATUS_NAMES.get(code, code)}")

    def shutdown(self) -> None:
        torch.cuda.synchronize(self.device)
        self.slots = []
        self.output_slots = []
        self.bulk = torch.empty(0, dtype=torch.uint8, device=self.device)
