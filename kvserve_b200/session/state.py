"""Session and receive-slot state machines (role of
kvsfuse-vllm0.30.0/mooncake/compression/state.py:14-72), with the legal
transitions made explicit: an illegal transition raises instead of leaving a
session or slot in an inconsistent state."""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum, auto
from typing import Any, Optional


class SessionState(Enum):
    PLANNED = auto()
    OPENING = auto()
    ACTIVE = auto()
    DRAINING = auto()
    COMPLETE = auto()
    FAILED = auto()
    CANCELLED = auto()


class ReceiveSlotState(Enum):
    FREE = auto()
    GRANTED = auto()
    RECEIVED = auto()
    DECODING = auto()
    WRITEBACK = auto()


TERMINAL = frozenset({SessionState.COMPLETE, SessionState.FAILED, SessionState.CANCELLED})

_SESSION_NEXT = {
    SessionState.PLANNED: {SessionState.OPENING, SessionState.ACTIVE, SessionState.FAILED, SessionState.CANCELLED},
    SessionState.OPENING: {SessionState.ACTIVE, SessionState.FAILED, SessionState.CANCELLED},
    SessionState.ACTIVE: {SessionState.DRAINING, SessionState.COMPLETE, SessionState.FAILED, SessionState.CANCELLED},
    SessionState.DRAINING: {SessionState.COMPLETE, SessionState.FAILED, SessionState.CANCELLED},
}
_SLOT_NEXT = {
    ReceiveSlotState.FREE: {ReceiveSlotState.GRANTED},
    ReceiveSlotState.GRANTED: {ReceiveSlotState.RECEIVED, ReceiveSlotState.FREE},
    ReceiveSlotState.RECEIVED: {ReceiveSlotState.DECODING, ReceiveSlotState.FREE},
    ReceiveSlotState.DECODING: {ReceiveSlotState.WRITEBACK, ReceiveSlotState.FREE},
    ReceiveSlotState.WRITEBACK: {ReceiveSlotState.FREE},
}


class IllegalTransition(RuntimeError):
    pass


@dataclass
class ReceiveSlot:
    slot_id: int
    offset: int = 0
    state: ReceiveSlotState = ReceiveSlotState.FREE
    chunk_id: Optional[int] = None
    owner: Optional[str] = None

    def move(self, new: ReceiveSlotState, chunk_id: Optional[int] = None, owner: Optional[str] = None) -> None:
        if new not in _SLOT_NEXT[self.state]:
            raise IllegalTransition(f"slot {self.slot_id}: {self.state.name} -> {new.name}")
        self.state = new
        if new is ReceiveSlotState.FREE:
            self.chunk_id, self.owner = None, None
        if chunk_id is not None:
            self.chunk_id = chunk_id
        if owner is not None:
            self.owner = owner


@dataclass
class _Session:
    transfer_id: str
    d_req_id: str
    state: SessionState = SessionState.PLANNED
    total_chunks: int = 0
    completed_chunks: int = 0
    error: Optional[str] = None
    nonce: str = ""
    valid_tokens_by_group: dict = field(default_factory=dict)
    deadline: float = float("inf")

    def move(self, new: SessionState) -> None:
        if self.state in TERMINAL or new not in _SESSION_NEXT.get(self.state, ()):
            raise IllegalTransition(f"session {self.transfer_id}: {self.state.name} -> {new.name}")
        self.state = new

    @property
    def done(self) -> bool:
        return self.state in TERMINAL


@dataclass
class ProducerSession(_Session):
    local_block_ids: list = field(default_factory=list)
    remote_block_ids: list = field(default_factory=list)
    remote_session: str = ""
    logical_block_count: int = 0
    inflight_chunks: int = 0
    send_meta: Any = None
    execution: Any = None
    remote_meta: Any = None     # the consumer's XferMetadata (its arena's IPC handle, slot geometry)


@dataclass
class ConsumerSession(_Session):
    block_ids: list = field(default_factory=list)
    logical_block_count: int = 0
    slots: list = field(default_factory=list)
    next_chunk: int = 0
    execution: Any = None
