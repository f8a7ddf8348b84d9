"""Summary of the transport's JSONL stats rows (role of the transport summary
of the reference's remote harness, tests/test_kvserve_remote.py:71-199).

Reads the rows :class:`~kvserve_b200.transport.nccl_transport.NcclTransport`
and the connectors append to ``KVSERVE_TRANSPORT_STATS_PATH`` (directions
``send``, ``recv``, ``credit_retry``, ``recv_credit``,
``recv_credit_release``, ``load_wait``, ``backpressure``) and reduces them
to per-direction counts, bytes, and p50 / p95 / max of the timing fields
(queue wait, ack, data-plane time, total; consumer receive wait; producer
backpressure wait), plus the credit retries and the share of blocked
submissions.

    python -m kvserve_b200.transport.stats_summary stats.jsonl [more.jsonl]
"""
from __future__ import annotations

import json
import math
import sys
from collections import defaultdict
from typing import Iterable

TIMINGS = {
    "send": ("queue_wait_s", "ack_s", "nccl_s", "total_s"),
    "recv": ("nccl_s", "total_s"),
    "load_wait": ("receive_wait_s", "start_load_total_s"),
    "backpressure": ("wait_s",),
}


def _pct(xs: list, q: float) -> float:
    """Nearest-rank percentile of a non-empty list."""
    s = sorted(xs)
    return s[min(len(s) - 1, max(0, math.ceil(q * len(s)) - 1))]


def read_rows(paths: Iterable[str]) -> list:
    rows = []
    for p in paths:
        with open(p, encoding="utf-8") as f:
            for line in f:
                line = line.strip()
                if line:
                    try:
                        rows.append(json.loads(line))
                    except json.JSONDecodeError:
                        continue      # a row cut by a crashed writer
    return rows


def summarize(rows: list) -> dict:
    by_dir: dict = defaultdict(list)
    for r in rows:
        by_dir[r.get("direction", "?")].append(r)
    out: dict = {"rows": len(rows), "directions": {}}
    for d, rs in sorted(by_dir.items()):
        s: dict = {"count": len(rs)}
        nbytes = [r["payload_bytes"] for r in rs if isinstance(r.get("payload_bytes"), (int, float))]
        if nbytes:
            s["payload_bytes"] = int(sum(nbytes))
        kinds: dict = defaultdict(int)
        for r in rs:
            if "kind" in r:
                kinds[str(r["kind"])] += 1
        if kinds:
            s["kinds"] = dict(kinds)
        for field in TIMINGS.get(d, ()):
            xs = [float(r[field]) for r in rs if isinstance(r.get(field), (int, float))]
            if xs:
                s[field] = {"p50_ms": round(1e3 * _pct(xs, 0.50), 3), "p95_ms": round(1e3 * _pct(xs, 0.95), 3),
                            "max_ms": round(1e3 * max(xs), 3)}
        if d == "backpressure":
            s["blocked_share"] = round(sum(1 for r in rs if r.get("blocked")) / len(rs), 4)
        out["directions"][d] = s
    send = out["directions"].get("send")
    if send and send.get("total_s") and send.get("payload_bytes"):
        out["send_throughput_MBps_at_p50"] = round(
            send["payload_bytes"] / send["count"] / max(1e-9, send["total_s"]["p50_ms"] / 1e3) / 1e6, 2)
    out["credit_retries"] = out["directions"].get("credit_retry", {}).get("count", 0)
    return out


def main(argv=None) -> None:
    paths = list(argv if argv is not None else sys.argv[1:])
    if not paths:
        raise SystemExit("usage: python -m kvserve_b200.transport.stats_summary stats.jsonl [...]")
    print(json.dumps(summarize(read_rows(paths)), indent=2))


if __name__ == "__main__":
    main()
