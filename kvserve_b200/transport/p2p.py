"""NVLink peer-memory KV channel (one prefill rank -> one decode rank).

The decode rank owns ``num_slots`` receive slots (each ``num_layers`` frames
of ``frame_stride`` bytes) and, per slot, a control block of u32 words

    [layer flags x num_layers][first token][token flag][credit][pad]

all in plain ``cudaMalloc`` memory exported through CUDA IPC.  The prefill rank maps
them and its fused encode kernel stores the packed frame straight into the
slot and release-stores the request sequence number into the flag; the
decode rank's fused decode kernel acquire-waits (bounded) on the flag and
writes the paged KV cache.  No NCCL send/recv is on this path — it replaces
the NCCL data plane of kvserve_v1/transport/nccl_transport.py:312-445.

In a single-process (colocated) deployment the same objects are used with
local pointers and the decode is stream-ordered after the encode.

Receiver credits (the role of kvserve_v1/transport/nccl_transport.py:519-560,
done on the device): a slot's ``credit`` word holds the sequence number of
the last request the decode rank has finished reading from it.  The decode
rank release-stores it (``store_release_u32``, system scope) once the ingest
kernels that read the slot have completed; before the prefill rank's encode
kernels store request ``seq`` into a slot, a one-thread kernel on the same
stream acquire-waits (bounded, over NVLink) until the credit reaches the
sequence number of the slot's previous request.  With ``num_slots`` slots the
prefill side runs up to ``num_slots`` requests ahead of the decode side's
ingest.

Slots are ``slot_stride`` bytes apart: the slot proper (``num_layers x
frame_stride``) and, with ``KVSERVE_SLOT_CANARIES=1``, a guard region that
:meth:`FrameReceiver.damaged_slots` checks for overruns (:mod:`.canary`).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from ..ops import ext
from .canary import GUARD_BYTES, canaries_enabled, damaged_slots, fill_guards


def ctrl_words(num_layers: int) -> int:
    """u32 words of one slot's control block."""
    return num_layers + 4


@dataclass
class ChannelHandles:
    slots: bytes
    flags: bytes
    slot_bytes: int
    num_slots: int
    num_layers: int
    frame_stride: int
    slot_stride: int = 0      # bytes between slots (slot_bytes plus a guard); 0 = slot_bytes


class FrameReceiver:
    """Decode-side receive slots + publish flags (device memory)."""

    def __init__(self, num_layers: int, frame_stride: int, num_slots: int = 1, device=None,
                 guard_bytes: Optional[int] = None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.num_layers, self.frame_stride, self.num_slots = num_layers, frame_stride, num_slots
        self.slot_bytes = num_layers * frame_stride
        self.guard_bytes = (GUARD_BYTES if canaries_enabled() else 0) if guard_bytes is None else int(guard_bytes)
        if self.guard_bytes % 256:
            raise ValueError("guard_bytes must keep slots 256-byte aligned")
        self.slot_stride = self.slot_bytes + self.guard_bytes
        with torch.cuda.device(self.device):
            self.slots_ptr = ext().dev_alloc(num_slots * self.slot_stride)
            # per slot: one publish flag per layer, the first token, its flag,
            # the credit word and one pad word
            self.flags_ptr = ext().dev_alloc(max(256, num_slots * ctrl_words(num_layers) * 4))
        self._closed = False
        if self.guard_bytes:
            fill_guards(self._slots_view(), num_slots, self.slot_stride, self.slot_bytes)

    def _slots_view(self) -> torch.Tensor:
        from ..ops import dtype_code
        return ext().tensor_from_ptr(self.slots_ptr, [self.num_slots * self.slot_stride], dtype_code(torch.uint8),
                                     self.device.index)

    def damaged_slots(self) -> list[int]:
        """Slots whose guard region was written (empty without guards);
        synchronises with the device."""
        if not self.guard_bytes:
            return []
        return damaged_slots(self._slots_view(), self.num_slots, self.slot_stride, self.slot_bytes)

    def slot_base(self, slot: int) -> int:
        return self.slots_ptr + slot * self.slot_stride

    def flags_base(self, slot: int) -> int:
        return self.flags_ptr + slot * ctrl_words(self.num_layers) * 4

    def token_ptr(self, slot: int) -> int:
        """[token value, token flag] of the slot's request."""
        return self.flags_base(slot) + self.num_layers * 4

    def credit_ptr(self, slot: int) -> int:
        """The slot's credit word (last sequence number read out of it)."""
        return self.flags_base(slot) + (self.num_layers + 2) * 4

    def handles(self) -> ChannelHandles:
        return ChannelHandles(ext().ipc_get_handle(self.slots_ptr), ext().ipc_get_handle(self.flags_ptr),
                              self.slot_bytes, self.num_slots, self.num_layers, self.frame_stride,
                              self.slot_stride)

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
            self.num_slots, self.slot_stride = local.num_slots, local.slot_stride
            return
        assert handles is not None
        with torch.cuda.device(self.device):
            self.slots_ptr = ext().ipc_open_handle(handles.slots)
            self.flags_ptr = ext().ipc_open_handle(handles.flags)
        self._opened = [self.slots_ptr, self.flags_ptr]
        self.slot_bytes, self.num_layers = handles.slot_bytes, handles.num_layers
        self.frame_stride, self.num_slots = handles.frame_stride, handles.num_slots
        self.slot_stride = handles.slot_stride or handles.slot_bytes

    def frame_ptr(self, slot: int, layer: int) -> int:
        return self.slots_ptr + slot * self.slot_stride + layer * self.frame_stride

    def flag_ptr(self, slot: int, layer: int) -> int:
        return self.flags_ptr + (slot * ctrl_words(self.num_layers) + layer) * 4

    def token_ptr(self, slot: int) -> int:
        return self.flags_ptr + (slot * ctrl_words(self.num_layers) + self.num_layers) * 4

    def credit_ptr(self, slot: int) -> int:
        return self.flags_ptr + (slot * ctrl_words(self.num_layers) + self.num_layers + 2) * 4

    def close(self) -> None:
        with torch.cuda.device(self.device):
            for p in self._opened:
                ext().ipc_close(p)
        self._opened = []
