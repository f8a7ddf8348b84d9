"""Tracing of the KV hand-off: NVTX ranges on the host and %globaltimer
stamps written by the fused kernels on the device.

* :func:`nvtx_range` marks host phases (each prefill layer, each encode
  launch, the ingest launch) for Nsight-style timelines.  On by default
  (``KVSERVE_NVTX=0`` turns it off); without a profiler attached a range
  costs a few hundred nanoseconds of host time.
* Stamps: with ``KVSERVE_TRACE=1`` the engine hands the encode and decode
  kernels a ``[layers, 4]`` int64 buffer; per layer the kernels record
  (``%globaltimer`` ns) the encode start, the moment the frame was published,
  the first decode CTA past the layer's flag and the last decode store
  (starts are kept as ``~t`` so the earliest CTA wins an atomic max).
  :func:`decode_stamps` turns the buffer into per-layer milliseconds and
  :func:`write_trace_row` appends them to the JSONL file named by
  ``KVSERVE_TRACE_FILE`` — the per-request stats rows of the reference's
  transport (kvserve_v1/transport/nccl_transport.py:447-463) with a
  device-side time line added.
"""
from __future__ import annotations

import contextlib
import json
import os
import time
from typing import Optional

import torch

_NVTX = os.environ.get("KVSERVE_NVTX", "1").strip().lower() not in {"0", "false", "no", "off"}


def trace_enabled() -> bool:
    return os.environ.get("KVSERVE_TRACE", "0").strip().lower() in {"1", "true", "yes", "on"}


@contextlib.contextmanager
def nvtx_range(name: str):
    if _NVTX and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


def nvtx_push(name: str) -> None:
    """Open a range (paired with :func:`nvtx_pop`; for loops whose body is
    too long for a ``with`` block)."""
    if _NVTX and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)


def nvtx_pop() -> None:
    if _NVTX and torch.cuda.is_available():
        torch.cuda.nvtx.range_pop()


def decode_stamps(raw: torch.Tensor) -> dict:
    """``raw`` int64 [L, 4] (host) -> per-layer times in ms relative to the
    earliest stamp on this GPU plus that base (ns), NaN where not stamped.
    Columns: encode_start, published, ingest_start, ingest_end."""
    u = raw.to(torch.int64).tolist()
    mask = (1 << 64) - 1
    rows = []
    for e0, e1, i0, i1 in u:
        vals = [(~e0) & mask if e0 else None, e1 & mask if e1 else None,
                (~i0) & mask if i0 else None, i1 & mask if i1 else None]
        rows.append(vals)
    present = [v for r in rows for v in r if v is not None]
    base = min(present) if present else 0
    ms = [[(v - base) / 1e6 if v is not None else float("nan") for v in r] for r in rows]
    return {"base_ns": base, "columns": ["encode_start", "published", "ingest_start", "ingest_end"],
            "layers_ms": ms}


def summarize_stamps(st: dict) -> dict:
    """Hand-off summary of one rank's stamps: first encode start to last
    publish (prefill side), first ingest start to last ingest end (decode
    side), in ms."""
    import math
    cols = list(zip(*st["layers_ms"])) if st["layers_ms"] else [[], [], [], []]
    fin = lambda xs: [x for x in xs if not math.isnan(x)]  # noqa: E731
    out = {}
    e0, e1, i0, i1 = (fin(c) for c in cols)
    if e0 and e1:
        out["encode_span_ms"] = round(max(e1) - min(e0), 4)
    if i0 and i1:
        out["ingest_span_ms"] = round(max(i1) - min(i0), 4)
    return out


def write_trace_row(row: dict, path: Optional[str] = None) -> None:
    path = path or os.environ.get("KVSERVE_TRACE_FILE")
    if not path:
        return
    row = dict(row, wall_time=time.time())
    with open(path, "a") as f:
        f.write(json.dumps(row) + "\n")
