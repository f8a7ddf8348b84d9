"""Tiered value pool: GPU HBM (fastest, smallest), pinned host memory, then
files on disk.  ``put`` lands in the first tier; when a tier is over its
byte budget the least recently used values move down one tier (a device to
host copy, or a host tensor written to disk); ``get`` promotes the value
back to the device tier.  A background thread performs disk writes so a put
never waits on the filesystem.  Counters are exported as Prometheus metrics
in a private registry (``pool.registry``).

``shared=True`` (needs ``disk_dir``) makes the directory the store that
several processes share — the engines of one node, or a scheduler process
that only looks keys up: every put is also written through to its file, and
``contains`` / ``get`` consult the directory for keys this process never
held.  Files are written under a temporary name and renamed, so a reader
sees a whole value or none."""
from __future__ import annotations

import os
import queue
import threading
from collections import OrderedDict
from typing import Any, Optional

import torch


class TieredKVPool:
    def __init__(self, device_bytes: int, host_bytes: int, disk_dir: Optional[str] = None, device=None,
                 shared: bool = False, disk_bytes: Optional[int] = None):
        if shared and not disk_dir:
            raise ValueError("a shared pool needs disk_dir")
        self.shared = shared
        # byte budget of the directory (None: unbounded); the oldest files go
        # first, whichever process wrote them
        self.disk_budget = None if disk_bytes is None else int(disk_bytes)
        self._disk_estimate = 0
        self.device = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
        self.budget = {"device": int(device_bytes), "host": int(host_bytes)}
        self.disk_dir = disk_dir
        if disk_dir:
            os.makedirs(disk_dir, exist_ok=True)
        self.tiers: dict[str, OrderedDict] = {"device": OrderedDict(), "host": OrderedDict()}
        self.used = {"device": 0, "host": 0}
        self.on_disk: dict[str, str] = {}
        self._lock = threading.RLock()
        self._disk_q: "queue.Queue[Optional[tuple[str, Any]]]" = queue.Queue()
        self._disk_inflight = 0
        self._pending_disk: dict[str, Any] = {}
        self._writer = threading.Thread(target=self._disk_loop, daemon=True, name="kvs-store-disk")
        self._writer.start()
        from prometheus_client import CollectorRegistry, Counter, Gauge
        self.registry = CollectorRegistry()
        self.m_hits = Counter("kvs_store_hits", "values served", ["tier"], registry=self.registry)
        self.m_miss = Counter("kvs_store_misses", "lookups that found nothing", registry=self.registry)
        self.m_evict = Counter("kvs_store_demotions", "values moved down a tier", ["tier"], registry=self.registry)
        self.m_bytes = Gauge("kvs_store_bytes", "bytes held", ["tier"], registry=self.registry)

    # ----------------------------------------------------------- helpers
    @staticmethod
    def _nbytes(v: Any) -> int:
        if isinstance(v, torch.Tensor):
            return v.numel() * v.element_size()
        if isinstance(v, (tuple, list)):
            return sum(TieredKVPool._nbytes(x) for x in v)
        if isinstance(v, dict):
            return sum(TieredKVPool._nbytes(x) for x in v.values())
        return 0

    @staticmethod
    def _to(v: Any, device: torch.device, pin: bool = False) -> Any:
        if isinstance(v, torch.Tensor):
            if device.type == "cpu":
                out = v.to("cpu", non_blocking=False)
                return out.pin_memory() if pin and torch.cuda.is_available() else out
            return v.to(device, non_blocking=True)
        if isinstance(v, (tuple, list)):
            return type(v)(TieredKVPool._to(x, device, pin) for x in v)
        if isinstance(v, dict):
            return {k: TieredKVPool._to(x, device, pin) for k, x in v.items()}
        return v

    def _path(self, key: str) -> str:
        return os.path.join(self.disk_dir, key.replace("/", "__") + ".pt")

    def _enqueue_disk(self, key: str, value: Any) -> None:
        with self._lock:
            self._pending_disk[key] = value
            self._disk_inflight += 1
        self._disk_q.put((key, value))

    def _disk_loop(self) -> None:
        while True:
            item = self._disk_q.get()
            if item is None:
                return
            try:
                self._write_disk(*item)
            finally:
                with self._lock:
                    self._disk_inflight -= 1

    def _write_disk(self, key: str, value: Any) -> None:
        path = self._path(key)
        tmp = f"{path}.{os.getpid()}.{threading.get_ident()}.tmp"
        torch.save(self._to(value, torch.device("cpu")), tmp)
        size = os.path.getsize(tmp)
        os.replace(tmp, path)
        with self._lock:
            if self._pending_disk.get(key) is value:
                self._pending_disk.pop(key)
                self.on_disk[key] = path
        if self.disk_budget is not None:
            self._disk_estimate += size
            if self._disk_estimate > self.disk_budget:
                self._prune_disk()

    def _prune_disk(self) -> None:
        """Delete the oldest value files until the directory holds at most
        90 % of its budget (files of other processes sharing it included)."""
        files = []
        for e in os.scandir(self.disk_dir):
            if e.name.endswith(".pt"):
                try:
                    st = e.stat()
                except FileNotFoundError:      # removed by another process meanwhile
                    continue
                files.append((st.st_mtime, st.st_size, e.path))
        total = sum(f[1] for f in files)
        target = int(0.9 * self.disk_budget)
        for _, size, path in sorted(files):
            if total <= target:
                break
            try:
                os.remove(path)
            except FileNotFoundError:
                pass
            total -= size
            with self._lock:
                for key in [k for k, p in self.on_disk.items() if p == path]:
                    self.on_disk.pop(key)
                self.m_evict.labels("disk").inc()
        self._disk_estimate = total

    def _insert(self, tier: str, key: str, value: Any) -> None:
        t = self.tiers[tier]
        if key in t:
            self.used[tier] -= self._nbytes(t.pop(key))
        t[key] = value
        self.used[tier] += self._nbytes(value)
        self._rebalance(tier)

    def _rebalance(self, tier: str) -> None:
        t = self.tiers[tier]
        while self.used[tier] > self.budget[tier] and len(t) > 0:
            key, value = t.popitem(last=False)
            self.used[tier] -= self._nbytes(value)
            self.m_evict.labels(tier).inc()
            if tier == "device":
                self._insert("host", key, self._to(value, torch.device("cpu"), pin=True))
            elif self.disk_dir and not (self.shared and key in self.on_disk):
                self._enqueue_disk(key, value)
        for name in ("device", "host"):
            self.m_bytes.labels(name).set(self.used[name])

    # ------------------------------------------------------------- API
    def put(self, key: str, value: Any) -> None:
        with self._lock:
            self._drop(key)
            dev = self._to(value, self.device)
            self._insert("device", key, dev)
            if self.shared and key not in self._pending_disk:
                self._enqueue_disk(key, dev)       # write through: other processes read the file

    def _drop(self, key: str) -> None:
        for tier in ("device", "host"):
            v = self.tiers[tier].pop(key, None)
            if v is not None:
                self.used[tier] -= self._nbytes(v)
        self._pending_disk.pop(key, None)
        path = self.on_disk.pop(key, None)
        if path and os.path.exists(path):
            os.remove(path)

    def contains(self, key: str) -> bool:
        with self._lock:
            if any(key in t for t in self.tiers.values()) or key in self._pending_disk or key in self.on_disk:
                return True
        return self.shared and os.path.exists(self._path(key))

    def tier_of(self, key: str) -> Optional[str]:
        with self._lock:
            for name, t in self.tiers.items():
                if key in t:
                    return name
            if key in self._pending_disk or key in self.on_disk:
                return "disk"
            return None

    def get(self, key: str) -> Optional[Any]:
        """The value on the device tier (promoted there), or None."""
        with self._lock:
            for name in ("device", "host"):
                t = self.tiers[name]
                if key in t:
                    self.m_hits.labels(name).inc()
                    if name == "device":
                        t.move_to_end(key)
                        return t[key]
                    value = t.pop(key)
                    self.used["host"] -= self._nbytes(value)
                    dev = self._to(value, self.device)
                    self._insert("device", key, dev)
                    return dev
            value = self._pending_disk.get(key)
            if value is None and key in self.on_disk:
                value = torch.load(self.on_disk[key], weights_only=True)
            elif value is None and self.shared and os.path.exists(self._path(key)):
                value = torch.load(self._path(key), weights_only=True)   # written by another process
                self.on_disk[key] = self._path(key)
            if value is None:
                self.m_miss.inc()
                return None
            self.m_hits.labels("disk").inc()
            if not self.shared:
                self._drop(key)
            dev = self._to(value, self.device)
            self._insert("device", key, dev)
            return dev

    def flush(self) -> None:
        """Wait until queued disk writes have finished."""
        done = threading.Event()
        while True:
            with self._lock:
                if not self._pending_disk and self._disk_inflight == 0:
                    return
            done.wait(0.01)

    def close(self) -> None:
        self._disk_q.put(None)
        self._writer.join(timeout=5)
