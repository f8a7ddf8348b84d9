"""Host-side fault injection for the transport control plane.

Failures are made on the host only (dropped or delayed control replies,
refused receiver credit); no GPU is ever made to fault or hang.  Rules come
from code or from ``KVSERVE_FAULTS``, a comma-separated list of
``drop_ack:<request_id>``, ``refuse_credit:<n>`` (refuse the next n credit
requests) and ``delay_ack_ms:<ms>``.
"""
from __future__ import annotations

import os
import threading
import time
from dataclasses import dataclass, field


@dataclass
class FaultInjector:
    drop_ack_ids: set = field(default_factory=set)
    refuse_credits: int = 0
    delay_ack_ms: float = 0.0
    _lock: threading.Lock = field(default_factory=threading.Lock)

    @classmethod
    def from_env(cls) -> "FaultInjector":
        f = cls()
        for rule in filter(None, (r.strip() for r in os.environ.get("KVSERVE_FAULTS", "").split(","))):
            key, _, val = rule.partition(":")
            if key == "drop_ack":
                f.drop_ack_ids.add(val)
            elif key == "refuse_credit":
                f.refuse_credits = int(val)
            elif key == "delay_ack_ms":
                f.delay_ack_ms = float(val)
            else:
                raise ValueError(f"unknown fault rule {rule!r}")
        return f

    def drop_ack(self, request_id: str) -> bool:
        return request_id in self.drop_ack_ids

    def refuse_credit(self, request_id: str) -> bool:
        with self._lock:
            if self.refuse_credits > 0:
                self.refuse_credits -= 1
                return True
        return False

    def maybe_delay(self) -> None:
        if self.delay_ack_ms > 0:
            time.sleep(self.delay_ack_ms / 1e3)
