"""Guard regions ("canaries") behind the receive slots of the NVLink channel.

With ``KVSERVE_SLOT_CANARIES=1`` every receive slot of a
:class:`~kvserve_b200.transport.p2p.FrameReceiver` is followed by a
``GUARD_BYTES`` region filled with ``GUARD_PATTERN`` when the slot memory is
created.  A producer whose frame overruns its slot (a wrong frame stride, a
layout mismatch between the peers, a kernel indexing bug) writes into the
guard instead of the next slot's frames; the decode side checks the guards
after each request (a few hundred bytes per slot read back to the host) and
fails the request naming the damaged slot.  The guards sit between slots, so
the frame layout inside a slot and the slot base alignment (256 bytes) are
unchanged.  This complements the per-frame checks of the decode kernel
(header magic, request sequence number, token count and layer: a stale or
foreign frame returns the bad-header status).

The helpers work on any ``uint8`` tensor (CPU or CUDA) holding
``num_slots`` slots of ``stride`` bytes whose first ``payload`` bytes are
the slot proper.
"""
from __future__ import annotations

import os

import torch

GUARD_BYTES = 256
GUARD_PATTERN = 0xA5


def canaries_enabled() -> bool:
    return os.environ.get("KVSERVE_SLOT_CANARIES", "0").strip().lower() in {"1", "true", "yes", "on"}


def _guards(buf: torch.Tensor, num_slots: int, stride: int, payload: int) -> torch.Tensor:
    if buf.dtype != torch.uint8 or buf.numel() < num_slots * stride or not 0 <= payload <= stride:
        raise ValueError("guard layout does not fit the buffer")
    return buf[: num_slots * stride].view(num_slots, stride)[:, payload:]


def fill_guards(buf: torch.Tensor, num_slots: int, stride: int, payload: int, pattern: int = GUARD_PATTERN) -> None:
    _guards(buf, num_slots, stride, payload).fill_(pattern)


def damaged_slots(buf: torch.Tensor, num_slots: int, stride: int, payload: int,
                  pattern: int = GUARD_PATTERN) -> list[int]:
    """Slots whose guard no longer holds the pattern."""
    g = _guards(buf, num_slots, stride, payload)
    if g.shape[1] == 0:
        return []
    bad = (g != pattern).any(dim=1)
    return [int(i) for i in torch.nonzero(bad.cpu()).flatten().tolist()]
