"""Worker registration service and transfer statistics (role of
kvsfuse-vllm0.30.0/mooncake/mooncake_utils.py:19-126 and stats.py:20-146).

Prefill workers register ``(engine_id, tp_rank) -> session endpoint`` with a
small FastAPI app (:func:`serve`, or ``python -m kvserve_b200.session.bootstrap``);
decode workers query it through :class:`BootstrapClient` to find the
producer of a request.  :class:`TransferStats` aggregates per-transfer durations, bytes,
chunk counts and failures the way the reference's connector stats do.
"""
from __future__ import annotations

import statistics
import threading
from dataclasses import dataclass, field
from typing import Optional


class Registry:
    """Thread-safe ``(engine_id, tp_rank) -> endpoint`` table."""

    def __init__(self):
        self._lock = threading.Lock()
        self._workers: dict[tuple[str, int], dict] = {}

    def register(self, engine_id: str, tp_rank: int, endpoint: str, tp_size: int = 1, **extra) -> None:
        with self._lock:
            self._workers[(engine_id, int(tp_rank))] = {"endpoint": endpoint, "tp_size": int(tp_size), **extra}

    def query(self, engine_id: str, tp_rank: Optional[int] = None):
        with self._lock:
            if tp_rank is not None:
                return self._workers.get((engine_id, int(tp_rank)))
            return {r: v for (e, r), v in self._workers.items() if e == engine_id}

    def unregister(self, engine_id: str) -> int:
        with self._lock:
            keys = [k for k in self._workers if k[0] == engine_id]
            for k in keys:
                del self._workers[k]
        return len(keys)


def make_app(registry: Optional[Registry] = None):
    """FastAPI app: ``POST /register``, ``GET /query``, ``DELETE /engine/{id}``."""
    from fastapi import Body, FastAPI, HTTPException

    reg = registry or Registry()
    app = FastAPI(title="kvserve-b200 bootstrap")

    @app.post("/register")
    def register(w: dict = Body(...)):
        for k in ("engine_id", "tp_rank", "endpoint"):
            if k not in w:
                raise HTTPException(422, f"missing field {k}")
        reg.register(str(w["engine_id"]), int(w["tp_rank"]), str(w["endpoint"]), int(w.get("tp_size", 1)))
        return {"ok": True}

    @app.get("/query")
    def query(engine_id: str, tp_rank: Optional[int] = None):
        out = reg.query(engine_id, tp_rank)
        if not out:
            raise HTTPException(404, f"no worker for {engine_id}")
        return out if tp_rank is not None else {str(k): v for k, v in out.items()}

    @app.delete("/engine/{engine_id:path}")
    def drop(engine_id: str):
        return {"removed": reg.unregister(engine_id)}

    app.state.registry = reg
    return app


class BootstrapClient:
    """HTTP client of :func:`make_app`'s service (prefill workers register,
    decode workers look up the session endpoint of a rank)."""

    def __init__(self, url: str, timeout_s: float = 5.0):
        self.url, self.timeout_s = url.rstrip("/"), timeout_s

    def register(self, engine_id: str, tp_rank: int, endpoint: str, tp_size: int = 1) -> None:
        import requests
        r = requests.post(f"{self.url}/register", json={"engine_id": engine_id, "tp_rank": int(tp_rank),
                                                        "endpoint": endpoint, "tp_size": int(tp_size)},
                          timeout=self.timeout_s)
        r.raise_for_status()

    def endpoint(self, engine_id: str, tp_rank: int) -> Optional[str]:
        """The registered endpoint of ``(engine_id, tp_rank)``; None when
        the service does not know it."""
        import requests
        r = requests.get(f"{self.url}/query", params={"engine_id": engine_id, "tp_rank": int(tp_rank)},
                         timeout=self.timeout_s)
        if r.status_code == 404:
            return None
        r.raise_for_status()
        return str(r.json()["endpoint"])

    def unregister(self, engine_id: str) -> int:
        import requests
        r = requests.delete(f"{self.url}/engine/{engine_id}", timeout=self.timeout_s)
        r.raise_for_status()
        return int(r.json()["removed"])


def serve(host: str = "127.0.0.1", port: int = 8998, registry: Optional[Registry] = None,
          timeout_s: float = 10.0):
    """Run the bootstrap service on a background thread; returns the
    uvicorn server (``server.should_exit = True`` stops it) and the thread."""
    import time

    import uvicorn
    server = uvicorn.Server(uvicorn.Config(make_app(registry), host=host, port=port, log_level="warning"))
    thread = threading.Thread(target=server.run, name="kvs-bootstrap", daemon=True)
    thread.start()
    deadline = time.monotonic() + timeout_s
    while not server.started:
        if not thread.is_alive() or time.monotonic() > deadline:
            raise RuntimeError(f"bootstrap service did not start on {host}:{port}")
        time.sleep(0.01)
    return server, thread


@dataclass
class TransferStats:
    durations_s: list = field(default_factory=list)
    bytes_transferred: list = field(default_factory=list)
    chunks: list = field(default_factory=list)
    failed: int = 0

    def record(self, duration_s: float, nbytes: int, chunks: int = 1) -> None:
        self.durations_s.append(float(duration_s))
        self.bytes_transferred.append(int(nbytes))
        self.chunks.append(int(chunks))

    def record_failure(self) -> None:
        self.failed += 1

    def aggregate(self, other: "TransferStats") -> "TransferStats":
        return TransferStats(self.durations_s + other.durations_s, self.bytes_transferred + other.bytes_transferred,
                             self.chunks + other.chunks, self.failed + other.failed)

    def reduce(self) -> dict:
        n = len(self.durations_s)
        if n == 0:
            return {"num_transfers": 0, "failed": self.failed}
        total_b = sum(self.bytes_transferred)
        total_t = sum(self.durations_s)
        return {"num_transfers": n, "failed": self.failed,
                "avg_duration_ms": 1e3 * total_t / n, "p50_duration_ms": 1e3 * statistics.median(self.durations_s),
                "total_mb": total_b / 2 ** 20, "avg_mb_per_transfer": total_b / n / 2 ** 20,
                "throughput_gbps": 8 * total_b / total_t / 1e9 if total_t > 0 else 0.0,
                "avg_chunks": sum(self.chunks) / n}


def main(argv=None) -> None:
    """``python -m kvserve_b200.session.bootstrap --host 0.0.0.0 --port 8998``"""
    import argparse

    import uvicorn
    ap = argparse.ArgumentParser(description="session endpoint registry for prefill and decode workers")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8998)
    a = ap.parse_args(argv)
    uvicorn.run(make_app(), host=a.host, port=a.port, log_level="warning")


if __name__ == "__main__":
    main()
