"""vLLM V1 KV connector over the chunked compression session: the decode
engine pulls the prompt KV chunk by chunk, the prefill engine encodes each
pulled chunk straight into the decode GPU's receive slot (role of the
in-tree MooncakeConnector, kvsfuse-vllm0.30.0/mooncake/mooncake_connector.py:
615-788 connector, 790-1087 scheduler side, 1090-3957 worker side).

Load it into vLLM with::

    KVTransferConfig(kv_connector="SessionKVConnector",
                     kv_connector_module_path="kvserve_b200.connector.session_kv_connector",
                     kv_role="kv_producer" | "kv_consumer", kv_ip=<prefill host>,
                     kv_connector_extra_config={"session_port": 26100, "num_slots": 4,
                                                "compression": {...runtime keys...}})

The ``compression`` object uses the runtime's keys
(``enable-compression-pipeline``, ``pipeline``, ``logical_blocks_per_chunk``,
the level keys, ...); both engines must use the same one.

Router contract (``kv_transfer_params``), the same shape as vLLM's own
pull-based connectors:

* prefill request: ``{"do_remote_decode": True, "transfer_id": T}``; the
  prefill engine's output carries ``{"do_remote_prefill": True,
  "transfer_id": T, "remote_host": h, "remote_port": p, "remote_tp_size": n,
  "remote_engine_id": e}``;
* decode request: that dict unchanged.

With ``bootstrap_url`` in the extra config (the service of
:mod:`kvserve_b200.session.bootstrap`), prefill workers register their
session endpoints under the engine id and decode workers look the prefill
rank up there; without it, or when the service does not know the engine,
the endpoint is ``remote_host`` and ``remote_port`` + rank.

Flow:

* prefill scheduler: ``request_finished`` keeps the blocks of a finished
  (length-capped) remote-decode request (``delay_free_blocks``) and queues a
  send for the worker; the next step's metadata registers it with the
  worker's :class:`~kvserve_b200.session.service.ProducerService`;
* decode scheduler: claims ``prompt - computed`` tokens as an asynchronous
  load, records the request's unhashed (new) blocks after allocation, and
  the next step's metadata opens a session;
* workers: each runs its session service on a thread of its own (ZeroMQ
  sockets stay in that thread); the prefill side's encode job is
  :class:`~kvserve_b200.session.gpu_jobs.RuntimeEncodeJob` over the
  compression runtime bound to vLLM's paged cache, the decode side's
  :class:`~kvserve_b200.session.gpu_jobs.RuntimeDecodeJob` decodes each
  chunk from its CUDA-IPC receive arena into the request's blocks;
* ``get_finished`` reports finished sends (the prefill engine frees the
  blocks) and finished loads (the decode engine schedules the request);
  a failed load reports its blocks through ``get_block_ids_with_load_errors``
  so vLLM recomputes them.

A decode engine that already holds a block-aligned prefix (prefix caching)
pulls only the suffix: the producer sends its last blocks and counts
tokens from the suffix start.

Tensor parallelism: prefill rank ``r`` serves on ``session_port + r``.  The
two engines may use different TP sizes (``prefill_tp_size`` /
``decode_tp_size`` in the extra config, defaults: this engine's size): the
KV-head transfer plan (:func:`~kvserve_b200.session.tp_plan.transfer_plan`)
gives each decode rank its heads as copies from the prefill ranks that hold
them, and every copy is one session (transfer id ``T#<decode rank>.<first
head>``) whose runtimes on both sides are bound to that head range of the
caches; a request is loaded (or sent) once all its copies have ended.  Equal
TP sizes are the one-copy case.
Finished sessions append a JSONL row to ``KVSERVE_SESSION_STATS_PATH``.
Engines on different nodes set ``inline_payloads``: the decode side exports
no CUDA IPC arena and each chunk's payload travels inside the protocol's
reply over the ZeroMQ connection.
"""
from __future__ import annotations

import json
import logging
import os
import queue
import re
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Optional

import torch

try:  # vLLM is only needed when the connector is used inside vLLM
    from vllm.distributed.kv_transfer.kv_connector.v1.base import (KVConnectorBase_V1, KVConnectorMetadata,
                                                                   KVConnectorRole)
except Exception:  # pragma: no cover - vLLM missing
    class KVConnectorBase_V1:  # type: ignore[no-redef]
        def __init__(self, *a, **k):
            pass

    class KVConnectorMetadata:  # type: ignore[no-redef]
        pass

    class KVConnectorRole:  # type: ignore[no-redef]
        SCHEDULER = 0
        WORKER = 1

log = logging.getLogger("kvserve_b200.session_connector")

DEFAULT_SESSION_PORT = 26100


@dataclass
class SendReq:
    request_id: str
    transfer_id: str
    block_ids: list
    num_tokens: int


@dataclass
class RecvReq:
    request_id: str
    transfer_id: str
    host: str
    port: int
    block_ids: list
    num_tokens: int
    engine_id: str = ""          # the prefill engine, for a bootstrap lookup


@dataclass
class SessionConnectorMetadata(KVConnectorMetadata):
    sends: list = field(default_factory=list)     # prompt KV complete after this step's forward
    recvs: list = field(default_factory=list)
    cancels: list = field(default_factory=list)   # registered sends whose request freed its blocks


def layer_index(name: str, fallback: int) -> int:
    """The layer number in a vLLM attention-layer name
    (``model.layers.7.self_attn.attn`` -> 7)."""
    nums = re.findall(r"\.(\d+)\.", f".{name}.")
    return int(nums[-1]) if nums else fallback


def kv_pair(t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(K, V) views ``[blocks, block_size, H, D]`` of one layer's paged cache
    in either vLLM layout (``[2, blocks, ...]`` or ``[blocks, 2, ...]``)."""
    if t.dim() != 5:
        raise ValueError(f"expected a 5-D paged KV cache, got {tuple(t.shape)}")
    if t.shape[0] == 2:
        return t[0], t[1]
    if t.shape[1] == 2:
        return t[:, 0], t[:, 1]
    raise ValueError(f"cannot find the K/V axis of a cache of shape {tuple(t.shape)}")


def write_session_stats(row: dict) -> None:
    path = os.environ.get("KVSERVE_SESSION_STATS_PATH")
    if not path:
        return
    try:
        with open(path, "a") as f:
            f.write(json.dumps(dict(row, wall_time=time.time()), sort_keys=True) + "\n")
    except OSError as exc:
        log.warning("cannot write session stats: %s", exc)


class ServiceThread(threading.Thread):
    """Owns one session service: builds it on its own thread (ZeroMQ sockets
    are single-threaded), runs queued commands against it and polls it."""

    def __init__(self, make_service: Callable[[], Any], device: Optional[torch.device] = None,
                 after_poll: Optional[Callable[[Any], None]] = None, poll_ms: int = 2):
        super().__init__(daemon=True, name="kvserve-session")
        self._make, self._device, self._after = make_service, device, after_poll
        self._poll_ms = poll_ms
        self._cmds: "queue.SimpleQueue" = queue.SimpleQueue()
        self._halt = threading.Event()
        self._ready = threading.Event()
        self.error: Optional[BaseException] = None
        self.service = None

    def submit(self, fn: Callable[[Any], None]) -> None:
        self._cmds.put(fn)

    def wait_ready(self, timeout: float = 60.0) -> None:
        if not self._ready.wait(timeout):
            raise TimeoutError("the session service did not start")
        if self.error is not None:
            raise RuntimeError(f"the session service failed to start: {self.error}")

    def run(self) -> None:
        try:
            if self._device is not None and self._device.type == "cuda":
                torch.cuda.set_device(self._device)
            self.service = self._make()
        except BaseException as exc:  # noqa: BLE001 - reported through wait_ready
            self.error = exc
            self._ready.set()
            return
        self._ready.set()
        while not self._halt.is_set():
            try:
                while True:
                    try:
                        fn = self._cmds.get_nowait()
                    except queue.Empty:
                        break
                    fn(self.service)
                self.service.poll(self._poll_ms)
                if self._after is not None:
                    self._after(self.service)
            except BaseException as exc:  # noqa: BLE001 - a broken service ends the thread, loudly
                log.exception("session service failed")
                self.error = exc
                break
        try:
            self.service.close()
        except Exception:  # noqa: BLE001
            pass

    def stop(self, timeout: float = 5.0) -> None:
        self._halt.set()
        if self.is_alive():
            self.join(timeout)


try:
    from vllm.distributed.kv_transfer.kv_connector.v1.metrics import KVConnectorStats
except Exception:  # pragma: no cover - vLLM missing
    @dataclass
    class KVConnectorStats:  # type: ignore[no-redef]
        data: dict = field(default_factory=dict)


@dataclass
class SessionTransferStats(KVConnectorStats):
    """Transfer telemetry of the session connector for vLLM's metrics
    logger (role of MooncakeKVConnectorStats,
    kvsfuse-vllm0.30.0/mooncake/stats.py:20-146): per interval, loads
    completed and failed, chunks, payload and raw bytes, load durations."""

    def __post_init__(self):
        for k in ("loads", "failed", "chunks", "payload_bytes", "data_bytes"):
            self.data.setdefault(k, 0)
        self.data.setdefault("load_ms", [])

    def reset(self):
        self.data = {}
        self.__post_init__()

    def aggregate(self, other: "KVConnectorStats") -> "KVConnectorStats":
        for k, v in other.data.items():
            if k == "load_ms":
                self.data["load_ms"] = list(self.data.get("load_ms", [])) + list(v)
            else:
                self.data[k] = self.data.get(k, 0) + v
        return self

    def reduce(self) -> dict:
        ms = sorted(self.data.get("load_ms", []))
        out = {k: self.data.get(k, 0) for k in ("loads", "failed", "chunks")}
        out["payload_MB"] = round(self.data.get("payload_bytes", 0) / 1e6, 3)
        if self.data.get("payload_bytes"):
            out["compression_ratio"] = round(self.data.get("data_bytes", 0) / self.data["payload_bytes"], 3)
        if ms:
            out["load_ms_avg"] = round(sum(ms) / len(ms), 3)
            out["load_ms_p50"] = round(ms[len(ms) // 2], 3)
            out["load_ms_max"] = round(ms[-1], 3)
        return out

    def is_empty(self) -> bool:
        return not (self.data.get("loads") or self.data.get("failed") or self.data.get("chunks"))


class _HelperProxy:
    """The service methods the connector calls, forwarded to a session helper
    process (:mod:`kvserve_b200.session.process`).  Send events stay in this
    process, keyed by transfer id."""

    def __init__(self, proc, events: dict):
        self.proc, self.events = proc, events
        self.finished: list = []

    def add_send(self, transfer_id, local_block_ids, num_tokens, send_meta=None):
        from ..session.process import AddSend
        if send_meta is not None:
            self.events[transfer_id] = send_meta
        self.proc.request(AddSend(transfer_id, local_block_ids, num_tokens, None))

    def open(self, endpoint, transfer_id, d_req_id, block_ids, num_tokens, block_size=16,
             logical_blocks_per_chunk=1):
        from ..session.process import Open
        self.proc.request(Open(endpoint, transfer_id, d_req_id, block_ids, num_tokens, block_size,
                               logical_blocks_per_chunk))

    def cancel(self, transfer_id, reason):
        from ..session.process import Abort
        self.proc.request(Abort(transfer_id, reason))

    abort = cancel

    def poll(self, timeout_ms: int = 0) -> int:
        """Run the helper's pending GPU jobs here and collect ended sessions
        (as objects shaped like the services' sessions)."""
        from types import SimpleNamespace

        from ..session.state import SessionState
        n = self.proc.serve_jobs(timeout_ms / 1000.0)
        if self.proc.done:
            for d in self.proc.done:
                self.events.pop(d.transfer_id, None)
                self.finished.append(SimpleNamespace(transfer_id=d.transfer_id, state=SessionState[d.state],
                                                     error=d.error, completed_chunks=d.completed_chunks,
                                                     total_chunks=d.total_chunks))
            self.proc.done.clear()
        if not self.proc.proc.is_alive():
            raise RuntimeError("the session helper process exited")
        return n

    def close(self) -> None:
        self.proc.stop()


class SessionKVConnector(KVConnectorBase_V1):
    def __init__(self, vllm_config, role, kv_cache_config=None):
        super().__init__(vllm_config, role, kv_cache_config)
        cfg = vllm_config.kv_transfer_config
        extra = dict(cfg.kv_connector_extra_config or {})
        self.is_producer = cfg.is_kv_producer
        self._block_size = vllm_config.cache_config.block_size
        self._host = str(extra.get("session_host") or cfg.kv_ip or "127.0.0.1")
        self._port = int(extra.get("session_port", DEFAULT_SESSION_PORT))
        self._num_slots = int(extra.get("num_slots", 4))
        # peers on different nodes: no CUDA IPC arena, payloads inline in the replies
        self._inline = bool(extra.get("inline_payloads", False))
        self._open_timeout_s = float(extra.get("open_timeout_s", 120.0))
        self._session_timeout_s = float(extra.get("session_timeout_s", 120.0))
        self._extra = extra
        # optional registry of session endpoints: prefill workers register,
        # decode workers look up the producer's rank instead of host:port+rank
        self._bootstrap_url = str(extra.get("bootstrap_url") or "")
        self._engine_id = str(extra.get("engine_id") or getattr(cfg, "engine_id", None) or
                              f"{self._host}:{self._port}")
        par = getattr(vllm_config, "parallel_config", None)
        if int(getattr(par, "data_parallel_size", 1) or 1) > 1:
            # data-parallel replicas share the engine id: each registers and
            # is named as its own replica (the role of the reference's
            # bootstrap by dp_rank, mooncake_connector.py:191-231)
            self._engine_id += f"/dp{int(getattr(par, 'data_parallel_rank', 0) or 0)}"
        self._endpoints: dict[tuple[str, int], str] = {}
        self._tp_size = int(getattr(vllm_config.parallel_config, "tensor_parallel_size", 1) or 1)
        self._tp_rank = 0
        # TP sizes of the two engines (heterogeneous TP: KV-head copies)
        self._p_tp = int(extra.get("prefill_tp_size", self._tp_size))
        self._d_tp = int(extra.get("decode_tp_size", self._tp_size))
        if (self._p_tp if cfg.is_kv_producer else self._d_tp) != self._tp_size:
            raise ValueError("prefill_tp_size / decode_tp_size must match this engine's tensor_parallel_size")
        total = getattr(getattr(vllm_config, "model_config", None), "get_total_num_kv_heads", None)
        self._num_kv_heads = int(extra.get("num_kv_heads") or (total() if callable(total) else 0))
        self._copies: list = []
        self._window_blocks = self.sliding_window_blocks(kv_cache_config)
        # scheduler state
        self._pending_sends: list[SendReq] = []
        self._pending_recvs: list[RecvReq] = []
        # worker state
        self._lock = threading.Lock()
        self._send_rid: dict[str, str] = {}          # copy transfer id -> prefill request id
        self._send_pending: dict[str, set] = {}      # prefill request id -> copy sessions not ended
        self._recv: dict[str, RecvReq] = {}          # copy transfer id -> load
        self._recv_pending: dict[str, set] = {}      # decode request id -> copy sessions not ended
        self._recv_started: dict[str, float] = {}
        self._stats = SessionTransferStats()
        self._svc_seen: dict[str, int] = {}
        self._done_sending: set[str] = set()
        self._done_recving: set[str] = set()
        self._finished_seen: set[str] = set()
        self._load_errors: set[int] = set()
        self._thread: Optional[ServiceThread] = None
        self._closers: list[Callable[[], None]] = []
        self._per_chunk = 1
        self._use_helper = bool(extra.get("session_process", os.environ.get("KVSERVE_SESSION_PROCESS", "0")
                                          .strip().lower() in {"1", "true", "yes", "on"}))
        self._device: Optional[torch.device] = None
        self._sends_this_step: list[SendReq] = []
        # scheduler: remote-decode requests -> (transfer id, prompt length,
        # blocks so far); transfer ids whose send was registered
        self._remote_decode: dict[str, tuple[str, int, list]] = {}
        self._registered: set[str] = set()
        self._pending_cancels: list[str] = []
        if role == KVConnectorRole.WORKER:
            try:
                from vllm.distributed.parallel_state import get_tensor_model_parallel_rank
                self._tp_rank = get_tensor_model_parallel_rank()
            except Exception:  # noqa: BLE001 - no TP group (tests)
                self._tp_rank = 0

    # ------------------------------------------------------------ helpers
    @staticmethod
    def sliding_window_blocks(kv_cache_config) -> int:
        """Trailing blocks of a request worth sending (0: all of them);
        see :func:`~kvserve_b200.connector.kv_groups.sliding_window_blocks`."""
        from .kv_groups import sliding_window_blocks
        return sliding_window_blocks(kv_cache_config, "SessionKVConnector")

    def runtime_config(self):
        from ..compression.runtime import CompressionConfig
        comp = self._extra.get("compression")
        if not isinstance(comp, dict):
            raise ValueError("SessionKVConnector needs kv_connector_extra_config['compression'] "
                             "with the runtime's keys")
        cfg = CompressionConfig.from_extra_config({"compression": comp})
        if not cfg.enabled:
            raise ValueError("SessionKVConnector runs the compression runtime; set enable-compression-pipeline")
        return cfg

    # ------------------------------------------------- heterogeneous TP
    def copies(self) -> list:
        """``(key, HeadCopy)`` of this worker: the KV-head ranges it sends
        (prefill) or receives (decode) under the transfer plan between the
        two TP groups; equal TP sizes give one full-shard copy."""
        from ..session.tp_plan import transfer_plan
        plan = transfer_plan(self._p_tp, self._d_tp, self._num_kv_heads)
        mine = [c for c in plan if (c.src_rank if self.is_producer else c.dst_rank) == self._tp_rank]
        return [(f"{c.dst_rank}.{c.dst_head}", c) for c in mine]

    @staticmethod
    def copy_tid(transfer_id: str, key: str) -> str:
        return f"{transfer_id}#{key}"

    @staticmethod
    def copy_key(copy_transfer_id: str) -> str:
        return copy_transfer_id.rsplit("#", 1)[1]

    def _global_first(self, c) -> int:
        from ..session.tp_plan import head_shard
        if self.is_producer:
            return head_shard(c.src_rank, self._p_tp, self._num_kv_heads).first + c.src_head
        return head_shard(c.dst_rank, self._d_tp, self._num_kv_heads).first + c.dst_head

    def _build_runtime(self, kv_caches: dict, execution: str, copy=None):
        """The compression runtime over ``copy``'s KV heads of vLLM's caches
        (all local heads without a copy).  Both peers build the runtime of a
        copy over the same global heads, as the shard of a virtual TP split
        into ``copy.heads``-head pieces, so head selection and signs agree."""
        from ..compression.runtime import CacheSpec, build_memory_plan, create_runtime
        cfg = self.runtime_config()
        specs, pairs = {}, {}
        for i, (name, t) in enumerate(kv_caches.items()):
            k, v = kv_pair(t)
            if copy is not None:
                h0 = copy.src_head if self.is_producer else copy.dst_head
                k, v = k[:, :, h0:h0 + copy.heads], v[:, :, h0:h0 + copy.heads]
            specs[name] = CacheSpec(layer_index(name, i), k.shape[1], k.shape[2], k.shape[3], k.dtype)
            pairs[name] = (k, v)
        dev = next(iter(kv_caches.values())).device
        if copy is None:
            tp_size, tp_rank = self._tp_size, self._tp_rank
        else:
            first = self._global_first(copy)
            if self._num_kv_heads % copy.heads or first % copy.heads:
                raise ValueError(f"KV-head copy {copy} does not align with {self._num_kv_heads} heads")
            tp_size, tp_rank = self._num_kv_heads // copy.heads, first // copy.heads
        plan = build_memory_plan(cfg, specs, tp_size=tp_size, tp_rank=tp_rank, device=dev)
        rt = create_runtime(plan, "NHD", 1, dev, execution=execution)
        rt.bind_kv_caches(pairs)
        return rt, cfg

    # ------------------------------------------------------------ worker
    def register_kv_caches(self, kv_caches: dict) -> None:
        from ..session.service import ConsumerService, ProducerService
        caches = {n: t for n, t in kv_caches.items() if isinstance(t, torch.Tensor) and t.numel() > 0}
        if not caches:
            raise ValueError("no paged KV caches to register")
        dev = next(iter(caches.values())).device
        self._device = dev
        if self._num_kv_heads <= 0:   # no model config: heads split (not replicated) over this TP group
            self._num_kv_heads = kv_pair(next(iter(caches.values())))[0].shape[2] * self._tp_size
        self._copies = self.copies()
        if self.is_producer:
            job = self.make_encode_job(caches)
            endpoint = f"tcp://*:{self._port + self._tp_rank}"
            if self._use_helper:
                make = lambda: self._helper("producer", {"endpoint": endpoint,  # noqa: E731
                                                         "open_timeout_s": self._open_timeout_s}, job)
            else:
                make = lambda: ProducerService(endpoint, job, self._open_timeout_s)  # noqa: E731
            self._thread = ServiceThread(make, dev, self._collect_sends)
        else:
            job, slot_bytes, handle = self.make_decode_job(caches)
            if self._inline:
                handle = b""
            name = f"kvs-d{self._tp_rank}-{os.getpid()}"
            if self._use_helper:
                def make():
                    proxy = self._helper("consumer", {"name": name, "num_slots": self._num_slots,
                                                      "slot_bytes": slot_bytes,
                                                      "session_timeout_s": self._session_timeout_s,
                                                      "arena_ipc_handle": handle}, job)
                    return proxy
                after = self._collect_recvs
            else:
                def make():
                    return ConsumerService(name, self._num_slots, slot_bytes, job, self._on_recv_done,
                                           self._session_timeout_s, arena_ipc_handle=handle)
                after = lambda svc: svc.finished.clear()  # noqa: E731
            self._thread = ServiceThread(make, dev, after)
        self._thread.start()
        self._thread.wait_ready()
        if self.is_producer and self._bootstrap_url:
            from ..session.bootstrap import BootstrapClient
            BootstrapClient(self._bootstrap_url).register(
                self._engine_id, self._tp_rank, f"tcp://{self._host}:{self._port + self._tp_rank}", self._tp_size)

    def _helper(self, role: str, cfg: dict, job) -> _HelperProxy:
        """Start the session helper process; its GPU jobs run ``job`` on the
        service thread of this process."""
        from types import SimpleNamespace

        from ..session.process import DecodeChunkJob, DrainSlotsJob, EncodeChunkJob, SessionProcess
        events: dict = {}

        def encode(j):
            sess = SimpleNamespace(transfer_id=j.transfer_id, remote_meta=j.remote_meta,
                                   send_meta=events.get(j.transfer_id), local_block_ids=j.local_block_ids,
                                   valid_tokens_by_group=j.valid_tokens_by_group)
            pull = SimpleNamespace(chunk_id=j.chunk_id, slot_id=j.slot_id, slot_offset=j.slot_offset,
                                   flag_index=j.flag_index, transfer_id=j.transfer_id)
            return job(sess, pull)

        def decode(j):
            sess = SimpleNamespace(transfer_id=j.transfer_id, block_ids=j.block_ids,
                                   valid_tokens_by_group=j.valid_tokens_by_group)
            slot = SimpleNamespace(slot_id=j.slot_id, offset=j.slot_offset)
            ready = SimpleNamespace(chunk_id=j.chunk_id, payload_bytes=j.payload_bytes)
            return job(sess, slot, ready)

        handlers = {DrainSlotsJob: lambda j: None}
        handlers[EncodeChunkJob if role == "producer" else DecodeChunkJob] = encode if role == "producer" \
            else decode
        return _HelperProxy(SessionProcess(role, cfg, handlers), events)

    def _collect_recvs(self, proxy) -> None:
        """Consumer with a helper process: ended sessions arrive as reports."""
        ended, proxy.finished[:] = list(proxy.finished), []
        for s in ended:
            self._on_recv_done(s)

    def make_encode_job(self, caches: dict):
        """The producer's ``encode_job``: per KV-head copy, the compression
        runtime bound to those heads of vLLM's paged cache, encoding each
        pulled chunk into the consumer's IPC-mapped slot; a session's copy
        is named by its transfer id."""
        from ..session.cpu_jobs import CpuEncodeJob
        from ..session.gpu_jobs import RuntimeEncodeJob
        jobs = {}
        for key, c in self._copies:
            rt, cfg = self._build_runtime(caches, "encode", c)
            self._per_chunk = cfg.logical_blocks_per_chunk
            job_cls = CpuEncodeJob if rt.device.type == "cpu" else RuntimeEncodeJob   # CPU engines: CPU runtime
            jobs[key] = job_cls(rt, self._block_size, cfg.logical_blocks_per_chunk)
            self._closers.append(jobs[key].close)
        return lambda session, pull: jobs[self.copy_key(session.transfer_id)](session, pull)

    def make_decode_job(self, caches: dict):
        """The consumer's ``decode_job`` (per KV-head copy, the runtime bound
        to those heads of its cache, reading one shared receive arena) plus
        the arena's slot size and CUDA-IPC handle."""
        from ..session.cpu_jobs import CpuDecodeJob, SharedArena
        from ..session.gpu_jobs import ReceiveArena, RuntimeDecodeJob, part_bytes
        built = [(key, *self._build_runtime(caches, "decode", c)) for key, c in self._copies]
        self._per_chunk = built[0][2].logical_blocks_per_chunk
        slot = 2 * max(part_bytes(rt) for _, rt, _ in built)
        cpu = built[0][1].device.type == "cpu"
        # CPU engines: a shared-memory arena and the CPU runtime's jobs
        arena = SharedArena(self._num_slots, slot) if cpu else ReceiveArena(self._num_slots, slot, built[0][1].device)
        self._closers.append(arena.close)
        job_cls = CpuDecodeJob if cpu else RuntimeDecodeJob
        jobs = {key: job_cls(rt, arena, self._block_size, cfg.logical_blocks_per_chunk) for key, rt, cfg in built}
        return (lambda session, slot, ready: jobs[self.copy_key(session.transfer_id)](session, slot, ready)), \
            arena.slot_bytes, arena.handle

    def start_load_kv(self, forward_context, **kwargs) -> None:
        meta = self._get_connector_metadata()
        if not isinstance(meta, SessionConnectorMetadata) or self._thread is None:
            return
        for tid in meta.cancels:
            for key, _ in self._copies:
                ct = self.copy_tid(tid, key)
                with self._lock:
                    rid = self._send_rid.pop(ct, None)
                    if rid is not None:
                        self._send_pending.pop(rid, None)
                self._thread.submit(lambda svc, ct=ct: svc.cancel(ct, "request not sent"))
        # sends are registered once this step's forward (which completes
        # their prompt KV) is enqueued: see wait_for_save
        self._sends_this_step = list(meta.sends)
        for r in meta.recvs:
            with self._lock:
                self._recv_started[r.request_id] = time.monotonic()
                self._recv_pending[r.request_id] = {self.copy_tid(r.transfer_id, k) for k, _ in self._copies}
                for key, _ in self._copies:
                    self._recv[self.copy_tid(r.transfer_id, key)] = r
            for key, c in self._copies:
                # the endpoint is looked up on the service thread: a bootstrap
                # query never stalls the model runner
                self._thread.submit(lambda svc, r=r, rank=c.src_rank, ct=self.copy_tid(r.transfer_id, key),
                                    pc=self._per_chunk: svc.open(
                    self._endpoint(r, rank), ct, r.request_id, [list(r.block_ids)], r.num_tokens,
                    block_size=self._block_size, logical_blocks_per_chunk=pc))

    def _endpoint(self, r: RecvReq, src_rank: int) -> str:
        """The session endpoint of prefill rank ``src_rank`` of ``r``'s
        engine: from the bootstrap service when one is configured and knows
        the engine (cached), else the request's host and port + rank."""
        if self._bootstrap_url and r.engine_id:
            key = (r.engine_id, src_rank)
            ep = self._endpoints.get(key)
            if ep is None:
                from ..session.bootstrap import BootstrapClient
                try:
                    ep = BootstrapClient(self._bootstrap_url).endpoint(r.engine_id, src_rank)
                except Exception as e:  # noqa: BLE001 - an unreachable registry: the direct address
                    log.warning("bootstrap lookup of %s failed: %s", key, e)
                if ep is not None:
                    self._endpoints[key] = ep
            if ep is not None:
                return ep
        return f"tcp://{r.host}:{r.port + src_rank}"

    def wait_for_save(self) -> None:
        """After the forward that completes the sends' prompt KV has been
        enqueued: register each send (one session per KV-head copy) with an
        event on the forward's stream, which the encode job waits for before
        it reads the blocks."""
        sends, self._sends_this_step = self._sends_this_step, []
        if not sends or self._thread is None:
            return
        ev = None
        if self._device is not None and self._device.type == "cuda":
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self._device))
        for snd in sends:
            cts = [self.copy_tid(snd.transfer_id, key) for key, _ in self._copies]
            with self._lock:
                self._send_pending[snd.request_id] = set(cts)
                for ct in cts:
                    self._send_rid[ct] = snd.request_id
            for ct in cts:
                self._thread.submit(lambda svc, ct=ct, snd=snd: svc.add_send(ct, [list(snd.block_ids)],
                                                                            snd.num_tokens, send_meta=ev))

    def _collect_sends(self, svc) -> None:
        """Producer thread: ended sessions; a request is sent once every
        copy's session has ended."""
        if not svc.finished:
            return
        ended, svc.finished[:] = list(svc.finished), []
        for s in ended:
            write_session_stats({"direction": "send", "transfer_id": s.transfer_id, "state": s.state.name,
                                 "chunks": s.completed_chunks, "error": s.error})
            with self._lock:
                rid = self._send_rid.pop(s.transfer_id, None)
                pending = self._send_pending.get(rid) if rid is not None else None
                if pending is not None:
                    pending.discard(s.transfer_id)
                    if not pending:
                        del self._send_pending[rid]
                        self._done_sending.add(rid)

    def _on_recv_done(self, s) -> None:
        """Consumer thread: one copy's load ended (complete, failed or timed
        out); the request is reported once all its copies have ended."""
        from ..session.state import SessionState
        with self._lock:
            r = self._recv.pop(s.transfer_id, None)
            if r is None:
                return
            if s.state is not SessionState.COMPLETE:
                self._load_errors.update(r.block_ids)
                self._stats.data["failed"] += 1
            self._stats.data["chunks"] += int(s.completed_chunks or 0)
            pending = self._recv_pending.get(r.request_id)
            if pending is not None:
                pending.discard(s.transfer_id)
                if not pending:
                    del self._recv_pending[r.request_id]
                    self._done_recving.add(r.request_id)
                    self._stats.data["loads"] += 1
                    t0 = self._recv_started.pop(r.request_id, None)
                    if t0 is not None:
                        self._stats.data["load_ms"].append(1e3 * (time.monotonic() - t0))
        write_session_stats({"direction": "recv", "transfer_id": s.transfer_id, "request_id": r.request_id,
                             "state": s.state.name, "chunks": s.completed_chunks, "total_chunks": s.total_chunks,
                             "error": s.error})

    def wait_for_layer_load(self, layer_name: str) -> None:
        return

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata, **kwargs) -> None:
        return

    def get_kv_connector_stats(self):
        """This interval's transfer telemetry (consumer side), then reset."""
        svc = self._thread.service if self._thread is not None else None
        with self._lock:
            st = self._stats
            if svc is not None and isinstance(getattr(svc, "stats", None), dict):
                for k in ("payload_bytes", "data_bytes"):
                    now = int(svc.stats.get(k, 0))
                    st.data[k] += now - self._svc_seen.get(k, 0)
                    self._svc_seen[k] = now
            self._stats = SessionTransferStats()
        return None if st.is_empty() else st

    @classmethod
    def build_kv_connector_stats(cls, data=None):
        return SessionTransferStats(data=dict(data or {}))

    def get_finished(self, finished_req_ids: set):
        if self._thread is not None and self._thread.error is not None:
            raise RuntimeError(f"session service failed: {self._thread.error}")
        with self._lock:
            self._finished_seen.update(finished_req_ids or ())
            # a send is reported once the scheduler has told this worker that
            # its request finished (vLLM's contract for delayed frees)
            sending = {r for r in self._done_sending if r in self._finished_seen}
            self._done_sending -= sending
            self._finished_seen -= sending
            recving, self._done_recving = self._done_recving, set()
        return (sending or None), (recving or None)

    def get_block_ids_with_load_errors(self) -> set:
        with self._lock:
            out, self._load_errors = self._load_errors, set()
        return out

    def shutdown(self) -> None:
        if self.is_producer and self._bootstrap_url and self._thread is not None and self._tp_rank == 0:
            from ..session.bootstrap import BootstrapClient
            try:
                BootstrapClient(self._bootstrap_url).unregister(self._engine_id)
            except Exception as e:  # noqa: BLE001 - the registry may be gone first
                log.warning("bootstrap unregister of %s failed: %s", self._engine_id, e)
        if self._thread is not None:
            self._thread.stop()
            self._thread = None
        for close in self._closers:
            try:
                close()
            except Exception:  # noqa: BLE001
                pass
        self._closers = []

    @classmethod
    def get_required_kvcache_layout(cls, vllm_config) -> Optional[str]:
        if vllm_config.model_config is None or vllm_config.model_config.use_mla:
            return None
        return "NHD"

    # ---------------------------------------------------------- scheduler
    def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
        params = getattr(request, "kv_transfer_params", None) or {}
        if self.is_producer or not params.get("do_remote_prefill") or "remote_port" not in params:
            return 0, False
        if int(params.get("remote_tp_size", self._p_tp)) != self._p_tp:
            # the copy plan is built for the configured prefill TP size: compute locally instead
            log.warning("request %s comes from a prefill engine of TP %s, configured for %s: not loaded",
                        request.request_id, params.get("remote_tp_size"), self._p_tp)
            return 0, False
        n = len(request.prompt_token_ids or []) - num_computed_tokens
        return (n, True) if n > 0 else (0, False)

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int) -> None:
        params = getattr(request, "kv_transfer_params", None) or {}
        if self.is_producer:
            if params.get("do_remote_decode") and params.get("transfer_id") \
                    and request.request_id not in self._remote_decode:
                self._remote_decode[request.request_id] = (str(params["transfer_id"]),
                                                           len(request.prompt_token_ids or []), [])
            return
        if not params.get("do_remote_prefill"):
            return
        params["do_remote_prefill"] = False      # one load per request
        if num_external_tokens <= 0:
            return
        get = getattr(blocks, "get_unhashed_block_ids_all_groups", None)
        ids = get()[0] if get is not None else blocks.get_block_ids()[0]
        if self._window_blocks and len(ids) > self._window_blocks:
            ids = ids[-self._window_blocks:]      # the rest fell out of the sliding window
        prompt = len(request.prompt_token_ids or [])
        full = -(-prompt // self._block_size)
        # the prompt's last `len(ids)` blocks are loaded; tokens from their start
        suffix = prompt - (full - len(ids)) * self._block_size
        self._pending_recvs.append(RecvReq(request.request_id, str(params["transfer_id"]),
                                           str(params.get("remote_host", self._host)), int(params["remote_port"]),
                                           list(ids), suffix, str(params.get("remote_engine_id", ""))))

    def build_connector_meta(self, scheduler_output):
        if self.is_producer and scheduler_output is not None:
            self._track_prefills(scheduler_output)
        # a send queued and cancelled before the worker saw it is dropped
        dropped = {s.transfer_id for s in self._pending_sends} & set(self._pending_cancels)
        meta = SessionConnectorMetadata(sends=[s for s in self._pending_sends if s.transfer_id not in dropped],
                                        recvs=self._pending_recvs,
                                        cancels=[t for t in self._pending_cancels if t not in dropped])
        self._pending_sends, self._pending_recvs, self._pending_cancels = [], [], []
        return meta

    def _track_prefills(self, so) -> None:
        """Queue a send for every remote-decode request whose prompt KV is
        complete after this step (its last prefill chunk is scheduled now)."""
        def step(rid, new_blocks, computed, resumed=False):
            tid, prompt, blocks = self._remote_decode[rid]
            blocks = list(new_blocks) if resumed else blocks + list(new_blocks)
            self._remote_decode[rid] = (tid, prompt, blocks)
            if tid not in self._registered and computed + so.num_scheduled_tokens.get(rid, 0) >= prompt:
                need = -(-prompt // self._block_size)
                self._pending_sends.append(SendReq(rid, tid, blocks[:need], prompt))
                self._registered.add(tid)
        for nr in so.scheduled_new_reqs:
            if nr.req_id in self._remote_decode:
                step(nr.req_id, nr.block_ids[0], nr.num_computed_tokens)
        cached = so.scheduled_cached_reqs
        resumed = getattr(cached, "resumed_req_ids", set()) or set()
        for i, rid in enumerate(cached.req_ids):
            if rid in self._remote_decode and cached.new_block_ids[i] is not None:
                step(rid, cached.new_block_ids[i][0], cached.num_computed_tokens[i], rid in resumed)
            elif rid in self._remote_decode:
                step(rid, [], cached.num_computed_tokens[i])

    def request_finished(self, request, block_ids):
        rid = request.request_id
        entry = self._remote_decode.pop(rid, None)
        if not self.is_producer or entry is None:
            return False, None
        tid = entry[0]
        status = getattr(request, "status", None)
        sendable = tid in self._registered and (status is None or
                                                getattr(status, "name", "") == "FINISHED_LENGTH_CAPPED")
        ids = block_ids[0] if block_ids and isinstance(block_ids[0], (list, tuple)) else list(block_ids or [])
        if not sendable or not ids:
            # aborted, stopped early or never prefilled: free now, send nothing
            if tid in self._registered:
                self._registered.discard(tid)
                self._pending_cancels.append(tid)
            return False, None
        self._registered.discard(tid)
        return True, {"do_remote_prefill": True, "do_remote_decode": False, "transfer_id": tid,
                      "remote_host": self._host, "remote_port": self._port, "remote_tp_size": self._tp_size,
                      "remote_num_tokens": entry[1], "remote_engine_id": self._engine_id}
