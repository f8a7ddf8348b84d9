"""vLLM V1 KV connector for disaggregated prefill/decode with compressed KV.

Load it into vLLM with::

    KVTransferConfig(kv_connector="CompressedKVConnector",
                     kv_connector_module_path="kvserve_b200.connector.compressed_kv_connector",
                     kv_role="kv_producer" | "kv_consumer", kv_rank=0 | 1, kv_parallel_size=2,
                     kv_ip=..., kv_port=25010,
                     kv_connector_extra_config={"compression": None | "default" | {...}})

Behaviour follows kvserve_v1/connector/compressed_kv_connector.py:

* scheduler (both roles): ``transfer_id`` from ``request.kv_transfer_params``
  (the router's stable key; falls back to the request id); the consumer claims
  ``prompt_len - 1 - computed`` external tokens loaded synchronously; the
  producer defers chunked prefills until the whole prompt KV exists;
  preempted requests are resumed.
* producer worker: ``save_kv_layer`` gathers the request's blocks per layer,
  ``wait_for_save`` stacks ``[L, 2, nb, bs, H, D]``, compresses with
  :class:`KVCompressionAdapter`, builds the wire and sends a bundle (raw send
  when compression is off or returns ``None``); sync by default, bounded
  async with ``KVSERVE_ASYNC_SEND`` / ``KVSERVE_MAX_INFLIGHT_BYTES``.
* consumer worker: ``start_load_kv`` drains the transport, consumes payloads
  of scheduled requests in arrival order (no head-of-line blocking), with a
  ``KVSERVE_LOAD_TIMEOUT_S`` deadline and fast failure on the transport's
  failure sentinel, decompresses, injects into the paged cache and returns
  receiver credit.
* the KV cache layout is forced to NHD.
"""
from __future__ import annotations

import json
import logging
import os
import time
from collections import defaultdict, deque
from dataclasses import dataclass, field
from typing import TYPE_CHECKING, Any, Optional

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

from ..compression.adapter import add_sentinel, is_compressed_layer_names, strip_sentinel
from ..compression.wire import CompressedWire, build_wire, restore_from_wire
from ..utils.kv_utils import (_kv_axis, extract_kv_from_layer_by_blocks, inject_kv_into_layer_by_blocks,
                              make_slot_mapping)

log = logging.getLogger("kvserve_b200.connector")


def _env_float(name: str, default: float) -> float:
    try:
        return float(os.environ.get(name, str(default)))
    except ValueError:
        return default


LOAD_TIMEOUT_S = _env_float("KVSERVE_LOAD_TIMEOUT_S", 60.0)
DEFAULT_MAX_CHUNK_BYTES = 512 * 1024 * 1024


def max_chunk_bytes() -> int:
    raw = os.environ.get("KVSERVE_MAX_NCCL_CHUNK_BYTES")
    try:
        v = int(raw) if raw else DEFAULT_MAX_CHUNK_BYTES
    except ValueError:
        v = DEFAULT_MAX_CHUNK_BYTES
    return v if v > 0 else DEFAULT_MAX_CHUNK_BYTES


def write_compression_stats(request_id: str, transfer_id: str, original: int, compressed: int) -> None:
    path = os.environ.get("KVSERVE_COMPRESSION_STATS_PATH")
    if not path or original <= 0 or compressed <= 0:
        return
    try:
        with open(path, "a") as f:
            f.write(json.dumps({"request_id": request_id, "transfer_id": transfer_id, "original_bytes": original,
                                "compressed_bytes": compressed}, sort_keys=True) + "\n")
    except OSError as exc:
        log.warning("cannot write compression stats: %s", exc)


@dataclass
class ReqMeta:
    request_id: str
    transfer_id: str
    token_ids: list
    block_ids: list
    slot_mapping: torch.Tensor


@dataclass
class CompressedKVConnectorMetadata(KVConnectorMetadata):
    requests: list = field(default_factory=list)

    def add_request(self, request_id: str, transfer_id: str, token_ids: list, block_ids: list,
                    block_size: int) -> None:
        self.requests.append(ReqMeta(request_id, transfer_id, list(token_ids), list(block_ids),
                                     make_slot_mapping(token_ids, block_ids, block_size)))


class CompressedKVConnector(KVConnectorBase_V1):
    def __init__(self, vllm_config, role, kv_cache_config=None):
        super().__init__(vllm_config, role, kv_cache_config)
        from .kv_groups import sliding_window_blocks
        sliding_window_blocks(kv_cache_config, "CompressedKVConnector")   # refuses several KV-cache groups
        cfg = vllm_config.kv_transfer_config
        self.is_producer = cfg.is_kv_producer
        self._block_size = vllm_config.cache_config.block_size
        self._async_send = os.environ.get("KVSERVE_ASYNC_SEND", "0").strip().lower() in {"1", "true", "yes", "on"}
        buf = max(1, int(cfg.kv_buffer_size))
        try:
            self._max_inflight_bytes = int(os.environ.get("KVSERVE_MAX_INFLIGHT_BYTES", str(buf)))
        except ValueError:
            self._max_inflight_bytes = buf
        self._requests_need_load: dict = {}
        self._request_transfer_ids: dict[str, str] = {}
        self.chunked_prefill: dict = {}
        self._worker_received_kv: dict = defaultdict(deque)
        self._layer_buffers: dict = {}
        self._num_kv_heads = vllm_config.model_config.get_num_kv_heads(vllm_config.parallel_config)
        self._head_size = vllm_config.model_config.get_head_size()
        self._num_layers = vllm_config.model_config.get_num_layers(vllm_config.parallel_config)
        self._model_name = os.path.basename(vllm_config.model_config.model.rstrip("/"))
        self._tp_rank, self._tp_size = 0, 1
        self._compressor = None
        self._compression_cfg = (cfg.kv_connector_extra_config or {}).get("compression")
        self._data_plane = (cfg.kv_connector_extra_config or {}).get("data_plane", "nccl")
        if role == KVConnectorRole.WORKER:
            from vllm.distributed.parallel_state import (get_tensor_model_parallel_rank,
                                                         get_tensor_model_parallel_world_size, get_world_group)
            local_rank = get_world_group().local_rank
            self._tp_rank = get_tensor_model_parallel_rank()
            self._tp_size = get_tensor_model_parallel_world_size()
            self._transport = self._build_transport(cfg, local_rank, self._tp_rank, self._data_plane)

    # ---- connector-owned memory, planned before KV sizing -----------------
    @classmethod
    def build_worker_memory_plan(cls, vllm_config, kv_cache_specs):
        """Plan this connector's GPU memory before the KV cache is sized
        (called by patched workers; stock vLLM can use
        :func:`~kvserve_b200.connector.memory_plan.adjusted_utilization`)."""
        from .memory_plan import plan_worker_memory
        extra = vllm_config.kv_transfer_config.kv_connector_extra_config or {}
        tp_size = int(getattr(vllm_config.parallel_config, "tensor_parallel_size", 1) or 1)
        tp_rank = 0
        try:
            from vllm.distributed.parallel_state import get_tensor_model_parallel_rank
            tp_rank = get_tensor_model_parallel_rank()
        except Exception:
            pass
        return plan_worker_memory(extra, kv_cache_specs, tp_rank, tp_size)

    def initialize_worker_memory(self, memory_plan) -> None:
        """Allocate exactly the planned memory after the KV cache exists."""
        from .memory_plan import WorkerMemory
        self._worker_memory = WorkerMemory(memory_plan)

    @classmethod
    def get_required_kvcache_layout(cls, vllm_config) -> Optional[str]:
        if vllm_config.model_config is None or vllm_config.model_config.use_mla:
            return None
        return "NHD"

    # ------------------------------------------------------------ worker
    def start_load_kv(self, forward_context, **kwargs) -> None:
        if self.is_producer:
            return
        for rid, items in self._transport.drain_received().items():
            self._worker_received_kv[rid].extend(items)
        meta = self._get_connector_metadata()
        if not isinstance(meta, CompressedKVConnectorMetadata):
            return
        pending = list(meta.requests)
        self._transport.set_expected_requests([r.transfer_id for r in pending])
        t0 = time.perf_counter()
        deadline = time.monotonic() + LOAD_TIMEOUT_S
        while pending:
            for rid, items in self._transport.drain_received().items():
                self._worker_received_kv[rid].extend(items)
            req = next((r for r in pending if self._worker_received_kv.get(r.transfer_id)), None)
            if req is None:
                if time.monotonic() > deadline:
                    for m in pending:
                        self._transport.record_stat({"direction": "load_wait", "kind": "timeout",
                                                     "request_id": m.transfer_id, "scheduler_request_id": m.request_id,
                                                     "receive_wait_s": time.perf_counter() - t0})
                    self._transport.set_expected_requests([])
                    raise TimeoutError("Timed out waiting for KV transfers: " +
                                       ", ".join(r.transfer_id for r in pending))
                time.sleep(0.005)
                continue
            pending.remove(req)
            names, payload = self._worker_received_kv[req.transfer_id].popleft()
            if not self._worker_received_kv[req.transfer_id]:
                self._worker_received_kv.pop(req.transfer_id, None)
            wait_s = time.perf_counter() - t0
            nbytes = self._transport.payload_nbytes(payload)
            try:
                if payload is None:
                    self._transport.record_stat({"direction": "load_wait", "kind": "failed",
                                                 "request_id": req.transfer_id,
                                                 "scheduler_request_id": req.request_id, "receive_wait_s": wait_s})
                    raise RuntimeError(f"KV transport failed for {req.transfer_id}")
                compressed = is_compressed_layer_names(names)
                if compressed:
                    names = strip_sentinel(names)
                    comp = self._get_compressor()
                    if comp is None or not isinstance(payload, dict) or not payload.get("__bundle__"):
                        raise RuntimeError(f"Invalid compressed KV payload for {req.transfer_id}")
                    stacked = comp.decompress(restore_from_wire(CompressedWire(
                        payload["meta"], payload["body_chunks"], payload["aux_tensors"])))
                    if stacked is None:
                        raise RuntimeError(f"KV decompression failed for {req.transfer_id}")
                else:
                    stacked = payload
                self.inject(forward_context, names, stacked, req)
                self._transport.record_stat({"direction": "load_wait", "kind": "compressed" if compressed else "raw",
                                             "request_id": req.transfer_id, "scheduler_request_id": req.request_id,
                                             "receive_wait_s": wait_s,
                                             "start_load_total_s": time.perf_counter() - t0})
            finally:
                if self._transport.device.type == "cuda":
                    torch.cuda.current_stream(self._transport.device).synchronize()
                self._transport.release_received(req.transfer_id, nbytes)
        self._transport.set_expected_requests([])

    @staticmethod
    def layer_cache(forward_context, name: str) -> Optional[torch.Tensor]:
        """The paged KV cache tensor of attention layer ``name``.  vLLM 0.22
        keeps one tensor per layer; older V1 releases kept a list with one
        cache per virtual engine, selected by ``forward_context.virtual_engine``."""
        layer = forward_context.no_compile_layers.get(name)
        kv = getattr(layer, "kv_cache", None) if layer is not None else None
        if isinstance(kv, (list, tuple)):
            kv = kv[getattr(forward_context, "virtual_engine", 0)] if kv else None
        if kv is None or kv.numel() == 0:
            return None
        return kv

    @classmethod
    def inject(cls, forward_context, names: list, stacked: torch.Tensor, req: ReqMeta) -> None:
        for i, name in enumerate(names):
            kv = cls.layer_cache(forward_context, name)
            if kv is not None:
                data = stacked[i].transpose(0, 1) if _kv_axis(kv) == 1 else stacked[i]
                inject_kv_into_layer_by_blocks(kv, data, req.block_ids, req.request_id)

    def wait_for_layer_load(self, layer_name: str) -> None:
        return

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata, **kwargs) -> None:
        if not self.is_producer:
            return
        meta = self._get_connector_metadata()
        if not isinstance(meta, CompressedKVConnectorMetadata):
            return
        blocks_first = _kv_axis(kv_layer) == 1
        for r in meta.requests:
            kv = extract_kv_from_layer_by_blocks(kv_layer, r.block_ids)
            # the wire carries [2, blocks, block_size, H, D] whatever the backend
            # (FlashInfer, vLLM's default on B200, stores [blocks, 2, ...])
            self._layer_buffers.setdefault(r.request_id, {})[layer_name] = \
                kv.transpose(0, 1).contiguous() if blocks_first else kv

    def wait_for_save(self) -> None:
        if not self.is_producer:
            return
        meta = self._get_connector_metadata()
        if not isinstance(meta, CompressedKVConnectorMetadata):
            return
        current = {r.request_id for r in meta.requests}
        for rid in set(self._layer_buffers) - current:
            self._layer_buffers.pop(rid, None)
        tids = [r.transfer_id for r in meta.requests]
        for r in meta.requests:
            layer_kv = self._layer_buffers.pop(r.request_id, None)
            if not layer_kv:
                continue
            names = sorted(layer_kv)
            stacked = torch.stack([layer_kv[n] for n in names], dim=0)
            self.send_stacked(r.request_id, r.transfer_id, names, stacked)
        if self._async_send:
            before = self._transport.pending_bytes()
            wait_s = self._transport.wait_for_below(self._max_inflight_bytes)
            if tids:
                self._transport.record_stat({"direction": "backpressure", "kind": "producer", "request_id": tids[0],
                                             "scheduled_requests": len(tids),
                                             "blocked": before > self._max_inflight_bytes,
                                             "pending_before_bytes": before,
                                             "pending_after_bytes": self._transport.pending_bytes(),
                                             "limit_bytes": self._max_inflight_bytes, "wait_s": wait_s})
        else:
            self._transport.wait_for_sent()

    def send_stacked(self, rid: str, transfer_id: str, names: list, stacked: torch.Tensor) -> None:
        comp = self._get_compressor()
        if comp is not None:
            t0 = time.monotonic()
            c = comp.compress(stacked, rid)
            if c is not None:
                w = build_wire(c, max_chunk_bytes())
                self._transport.send_bundle(transfer_id, add_sentinel(names), w.meta, w.body_chunks, w.aux_tensors)
                write_compression_stats(rid, transfer_id, stacked.numel() * stacked.element_size(), w.nbytes)
                comp.update_controller(rid, (time.monotonic() - t0) * 1e3)
                return
            log.warning("compression returned None for %s; sending raw", rid)
        self._transport.send(transfer_id, names, stacked)

    def get_finished(self, finished_req_ids: set):
        return None, None

    def shutdown(self) -> None:
        t = getattr(self, "_transport", None)
        if self.is_producer and t is not None:
            t.wait_for_sent()

    # ---------------------------------------------------------- scheduler
    def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
        if self.is_producer:
            return 0, False
        n = len(request.prompt_token_ids) - 1 - num_computed_tokens
        return (n, False) if n > 0 else (0, False)

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int) -> None:
        self._resolve_transfer_id(request.request_id, request)
        if not self.is_producer and num_external_tokens > 0:
            self._requests_need_load[request.request_id] = (request, blocks.get_block_ids()[0])

    def build_connector_meta(self, scheduler_output):
        meta = CompressedKVConnectorMetadata()
        for nr in scheduler_output.scheduled_new_reqs:
            if self.is_producer:
                n = scheduler_output.num_scheduled_tokens[nr.req_id] + nr.num_computed_tokens
                prompt = nr.prompt_token_ids or []
                if n < len(prompt):
                    self.chunked_prefill[nr.req_id] = (nr.block_ids[0], prompt)
                    continue
                meta.add_request(nr.req_id, self._resolve_transfer_id(nr.req_id), prompt, nr.block_ids[0],
                                 self._block_size)
            elif nr.req_id in self._requests_need_load:
                meta.add_request(nr.req_id, self._resolve_transfer_id(nr.req_id), nr.prompt_token_ids or [],
                                 nr.block_ids[0], self._block_size)
                self._requests_need_load.pop(nr.req_id)
        cached = scheduler_output.scheduled_cached_reqs
        resumed_ids = getattr(cached, "resumed_req_ids", set())
        for i, rid in enumerate(cached.req_ids):
            computed = cached.num_computed_tokens[i]
            new_blocks = cached.new_block_ids[i]
            resumed = rid in resumed_ids
            if self.is_producer:
                if rid not in self.chunked_prefill or new_blocks is None:
                    continue
                n = scheduler_output.num_scheduled_tokens[rid] + computed
                blocks = new_blocks[0] if resumed else self.chunked_prefill[rid][0] + new_blocks[0]
                prompt = self.chunked_prefill[rid][1]
                if n < len(prompt):
                    self.chunked_prefill[rid] = (blocks, prompt)
                    continue
                meta.add_request(rid, self._resolve_transfer_id(rid), prompt, blocks, self._block_size)
                self.chunked_prefill.pop(rid, None)
                continue
            if not resumed:
                break
            if rid in self._requests_need_load and new_blocks is not None:
                request, _ = self._requests_need_load.pop(rid)
                meta.add_request(rid, self._resolve_transfer_id(rid, request),
                                 request.all_token_ids[:computed + 1], new_blocks[0], self._block_size)
        return meta

    def request_finished(self, request, block_ids: list):
        self.chunked_prefill.pop(request.request_id, None)
        self._request_transfer_ids.pop(request.request_id, None)
        if not self.is_producer:
            self._requests_need_load.pop(request.request_id, None)
        return False, None

    # ----------------------------------------------------------- internal
    def _get_compressor(self):
        if self._compression_cfg is None:
            return None
        if self._compressor is None:
            from ..compression.adapter import KVCompressionAdapter
            self._compressor = KVCompressionAdapter(self._compression_cfg, self._num_kv_heads, self._head_size,
                                                    self._model_name, self._tp_rank, self._tp_size,
                                                    num_layers=self._num_layers)
        return self._compressor

    def _resolve_transfer_id(self, request_id: str, request=None) -> str:
        if request is not None:
            params = getattr(request, "kv_transfer_params", None)
            if params and params.get("transfer_id"):
                self._request_transfer_ids[request_id] = str(params["transfer_id"])
        return self._request_transfer_ids.get(request_id, request_id)

    @staticmethod
    def _build_transport(cfg, local_rank: int = 0, channel_rank: int = 0, data_plane: str = "nccl"):
        from ..transport.nccl_transport import NcclTransport
        return NcclTransport(cfg.is_kv_producer, cfg.kv_ip, cfg.kv_port, local_rank, channel_rank,
                             max(1, int(cfg.kv_buffer_size)), data_plane=data_plane)
