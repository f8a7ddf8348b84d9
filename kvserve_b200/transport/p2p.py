"""NVLink peer-memory KV channel (one prefill rank -> one decode rank).

The decode rank owns ``num_slots`` receive slots (each ``num_layers`` frames
of ``frame_stride`` bytes) and one u32 publish flag per (slot, layer), all in
plain ``cudaMalloc`` memory exported through CUDA IPC.  The prefill rank maps
them and its fused encode kernel stores the packed frame straight into the
slot and release-stores the request sequence number into the flag; the
decode rank's fused decode kernel acquire-waits (bounded) on the flag and
writes the paged KV cache.  No NCCL send/recv is on this path — it replaces
the NCCL data plane of kvserve_v1/transport/nccl_transport.py:312-445.

In a single-process (colocated) deployment the same objects are used with
local pointers and the decode is stream-ordered after the encode.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from ..ops import ext


@dataclass
class ChannelHandles:
    slots: bytes
    flags: bytes
    slot_bytes: int
    num_slots: int
    num_layers: int
    frame_stride: int


class FrameReceiver:
    """Decode-side receive slots + publish flags (device memory)."""

    def __init__(self, num_layers: int, frame_stride: int, num_slots: int = 1, device=None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.num_layers, self.frame_stride, self.num_slots = num_layers, frame_stride, num_slots
        self.slot_bytes = num_layers * frame_stride
        with torch.cuda.device(self.device):
            self.slots_ptr = ext().dev_alloc(num_slots * self.slot_bytes)
            # per slot: one publish flag per layer, then the first token and its flag
            self.flags_ptr = ext().dev_alloc(max(256, num_slots * (num_layers + 2) * 4))
        self._closed = False

    def slot_base(self, slot: int) -> int:
        return self.slots_ptr + slot * self.slot_bytes

    def flags_base(self, slot: int) -> int:
        return self.flags_ptr + slot * (self.num_layers + 2) * 4

    def token_ptr(self, slot: int) -> int:
        """[token value, token flag] of the slot's request."""
        return self.flags_base(slot) + self.num_layers * 4

    def handles(self) -> ChannelHandles:
        return ChannelHandles(ext().ipc_get_handle(self.slots_ptr), ext().ipc_get_handle(self.flags_ptr),
                              self.slot_bytes, self.num_slots, self.num_layers, self.frame_stride)

    def flags_view(self, slot: int) -> torch.Tensor:
        from ..ops import dtype_code
        return ext().tensor_from_ptr(self.flags_base(slot), [self.num_layers], dtype_code(torch.int32),
                                     self.device.index)

    def close(self) -> None:
        if not self._closed:
            with torch.cuda.device(self.device):
                ext().dev_free(self.slots_ptr)
                ext().dev_free(self.flags_ptr)
            self._closed = True


class FrameSender:
    """Prefill-side view of a receiver: peer pointers opened from IPC handles
    (or the receiver's own pointers when colocated)."""

    def __init__(self, handles: Optional[ChannelHandles] = None, local: Optional[FrameReceiver] = None,
                 device=None):
        self._opened: list[int] = []
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if local is not None:
            self.slots_ptr, self.flags_ptr = local.slots_ptr, local.flags_ptr
            self.slot_bytes, self.num_layers, self.frame_stride = local.slot_bytes, local.num_layers, local.frame_stride
            self.num_slots = local.num_slots
            return
        assert handles is not None
        with torch.cuda.device(self.device):
            self.slots_ptr = ext().ipc_open_handle(handles.slots)
            self.flags_ptr = ext().ipc_open_handle(handles.flags)
        self._opened = [self.slots_ptr, self.flags_ptr]
        self.slot_bytes, self.num_layers = handles.slot_bytes, handles.num_layers
        self.frame_stride, self.num_slots = handles.frame_stride, handles.num_slots

    def frame_ptr(self, slot: int, layer: int) -> int:
        return self.slots_ptr + slot * self.slot_bytes + layer * self.frame_stride

    def flag_ptr(self, slot: int, layer: int) -> int:
        return self.flags_ptr + (slot * (self.num_layers + 2) + layer) * 4

    def token_ptr(self, slot: int) -> int:
        return self.flags_ptr + (slot * (self.num_layers + 2) + self.num_layers) * 4

    def close(self) -> None:
        with torch.cuda.device(self.device):
            for p in self._opened:
                ext().ipc_close(p)
        self._opened = []
