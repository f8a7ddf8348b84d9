"""vLLM V1 KV connector over the shared prefix KV store (role of the
MooncakeStoreConnector, kvsfuse-vllm0.30.0/mooncake/store/connector.py:
125-411 with its scheduler.py / worker.py): every prompt's KV is saved per
chunk of blocks under its chained prefix hash, and a later request whose
prompt starts with a stored prefix loads those chunks instead of computing
them.

Load it into vLLM with::

    KVTransferConfig(kv_connector="StoreKVConnector",
                     kv_connector_module_path="kvserve_b200.connector.store_kv_connector",
                     kv_role="kv_both",
                     kv_connector_extra_config={"store": {"dir": "/dev/shm/kvs-store",
                                                          "device_bytes": 8 << 30, "host_bytes": 32 << 30,
                                                          "disk_bytes": 256 << 30, "blocks_per_chunk": 16},
                                                "compression": None | <modular profile>})

The store is a :class:`~kvserve_b200.store.pool.TieredKVPool` in shared mode:
each worker keeps hot chunks on its GPU and in pinned host memory and
writes every chunk through to ``store.dir``; the scheduler (often another
process) and other engines on the node look chunks up in that directory.
With ``compression`` the chunks are stored in the modular pipeline's wire
form (e.g. Hadamard + 4-bit), which is what the reference store lacks.

Flow:

* scheduler: ``get_num_new_matched_tokens`` counts the stored prefix chunks
  of the prompt beyond the locally computed tokens (keeping at least the
  last prompt token to compute) and claims them as a synchronous load;
  ``update_state_after_alloc`` records the request's blocks; each step's
  metadata carries the loads and the saves (requests whose prompt finishes
  in this step);
* worker: ``start_load_kv`` copies the chunks into the request's blocks
  before the forward (chunks the engine already holds are skipped);
  ``wait_for_save`` gathers the finished prompts' blocks after the forward
  (same stream) and puts each new chunk; a chunk that vanished between
  lookup and load is reported through ``get_block_ids_with_load_errors``.

Tensor parallelism: each TP rank stores its own head shard under a
rank-qualified key (:class:`~kvserve_b200.store.layout.RankLocalLayout`);
the scheduler looks up rank 0's keys.
"""
from __future__ import annotations

import logging
import os
import re
from dataclasses import dataclass, field
from typing import Optional

import torch

from .session_kv_connector import (KVConnectorBase_V1, KVConnectorMetadata, KVConnectorRole, KVConnectorStats,
                                   layer_index)

log = logging.getLogger("kvserve_b200.store_connector")


@dataclass
class StoreLoad:
    request_id: str
    token_ids: list
    block_ids: list
    first_block: int      # blocks already present locally
    num_tokens: int       # prefix tokens that must be in place afterwards


@dataclass
class StoreSave:
    request_id: str
    token_ids: list
    block_ids: list


@dataclass
class StoreStats(KVConnectorStats):
    """Per-interval store telemetry for vLLM's metrics logger: prefix tokens
    loaded, chunks saved, chunks that had vanished at load time."""

    def __post_init__(self):
        for k in ("loaded_tokens", "saved_chunks", "load_errors"):
            self.data.setdefault(k, 0)

    def reset(self):
        self.data = {}
        self.__post_init__()

    def aggregate(self, other: "KVConnectorStats") -> "KVConnectorStats":
        for k, v in other.data.items():
            self.data[k] = self.data.get(k, 0) + v
        return self

    def reduce(self) -> dict:
        return {k: self.data.get(k, 0) for k in ("loaded_tokens", "saved_chunks", "load_errors")}

    def is_empty(self) -> bool:
        return not any(self.data.get(k) for k in ("loaded_tokens", "saved_chunks", "load_errors"))


@dataclass
class StoreConnectorMetadata(KVConnectorMetadata):
    loads: list = field(default_factory=list)
    saves: list = field(default_factory=list)


class StoreKVConnector(KVConnectorBase_V1):
    def __init__(self, vllm_config, role, kv_cache_config=None):
        super().__init__(vllm_config, role, kv_cache_config)
        from .kv_groups import sliding_window_blocks
        if sliding_window_blocks(kv_cache_config, "StoreKVConnector"):
            # stored chunks are whole prompt prefixes, but blocks that left the
            # window hold stale KV: a shorter request reusing them would read it
            raise ValueError("StoreKVConnector keeps whole prompt prefixes; sliding-window KV-cache groups "
                             "free blocks outside the window, so their chunks can not be stored")
        extra = dict(vllm_config.kv_transfer_config.kv_connector_extra_config or {})
        st = dict(extra.get("store") or {})
        self._dir = st.get("dir")
        if not self._dir:
            raise ValueError("StoreKVConnector needs kv_connector_extra_config['store']['dir']")
        self._device_bytes = int(st.get("device_bytes", 1 << 30))
        self._host_bytes = int(st.get("host_bytes", 4 << 30))
        self._disk_bytes = int(st["disk_bytes"]) if st.get("disk_bytes") else None
        self._bpc = int(st.get("blocks_per_chunk", 16))
        self._block_size = vllm_config.cache_config.block_size
        self._compression = extra.get("compression")
        model = getattr(getattr(vllm_config, "model_config", None), "model", "model") or "model"
        self._model = re.sub(r"[^A-Za-z0-9_.-]", "_", os.path.basename(str(model).rstrip("/")))
        self._salt = str(st.get("salt", self._model)).encode()
        self._tp_size = int(getattr(vllm_config.parallel_config, "tensor_parallel_size", 1) or 1)
        self._tp_rank = 0
        self._store = None           # worker: KVStoreConnector over this rank's shard
        self._lookup_store = None    # scheduler: rank 0's keys, directory only
        self._layers: list = []
        # scheduler state
        self._pending_loads: list[StoreLoad] = []
        self._prefill: dict[str, tuple[list, list]] = {}   # request -> (token ids, blocks so far)
        self._pending_saves: list[StoreSave] = []
        self._local_hit: dict[str, int] = {}
        self._load_errors: set = set()
        self._errors_total = 0
        self._stats_seen: dict = {}
        self.stats = {"lookups": 0, "hit_tokens": 0, "loaded_tokens": 0, "saved_chunks": 0}
        if role == KVConnectorRole.WORKER:
            try:
                from vllm.distributed.parallel_state import get_tensor_model_parallel_rank
                self._tp_rank = get_tensor_model_parallel_rank()
            except Exception:  # noqa: BLE001 - no TP group (tests)
                self._tp_rank = 0

    # ------------------------------------------------------------ helpers
    def _make_store(self, rank: int, device, pool_bytes: tuple, compression=None, heads: int = 0,
                    head_size: int = 0, layers: Optional[int] = None):
        from ..store.connector import KVStoreConnector
        from ..store.layout import RankLocalLayout
        from ..store.pool import TieredKVPool
        pool = TieredKVPool(pool_bytes[0], pool_bytes[1], disk_dir=self._dir, device=device, shared=True,
                            disk_bytes=self._disk_bytes)
        return KVStoreConnector(pool, self._block_size, self._bpc, RankLocalLayout(self._model, rank, self._tp_size),
                                compression, heads, head_size, layers, self._salt)

    def _lookup(self, token_ids: list) -> int:
        if self._lookup_store is None:     # keys only: no memory tiers, no codec
            self._lookup_store = self._make_store(0, "cpu", (0, 0))
        return self._lookup_store.lookup(token_ids)

    # ---------------------------------------------------------- scheduler
    def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
        prompt = list(request.prompt_token_ids or [])
        self.stats["lookups"] += 1
        hit = self._lookup(prompt)
        # the last prompt token is always computed (it yields the next token)
        chunk = self._block_size * self._bpc
        hit = min(hit, (len(prompt) - 1) // chunk * chunk)
        n = hit - num_computed_tokens
        if n <= 0:
            return 0, False
        self.stats["hit_tokens"] += n
        # the scheduler sets the request's computed count after allocation:
        # remember the local prefix-cache hit for update_state_after_alloc
        self._local_hit[request.request_id] = num_computed_tokens
        return n, False

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int) -> None:
        computed = self._local_hit.pop(request.request_id, 0)
        if num_external_tokens <= 0 or blocks is None:
            return
        ids = list(blocks.get_block_ids()[0])
        prompt = list(request.prompt_token_ids or [])
        self._pending_loads.append(StoreLoad(request.request_id, prompt, ids, computed // self._block_size,
                                             computed + num_external_tokens))

    def build_connector_meta(self, scheduler_output):
        if scheduler_output is not None:
            self._track_prefills(scheduler_output)
        meta = StoreConnectorMetadata(loads=self._pending_loads, saves=self._pending_saves)
        self._pending_loads, self._pending_saves = [], []
        return meta

    def _track_prefills(self, so) -> None:
        """Queue a save for every request whose prompt is complete after this
        step (the step that schedules its last prefill tokens)."""
        def step(rid, prompt, new_blocks, computed, resumed=False):
            toks, blocks = self._prefill.get(rid, (prompt, []))
            blocks = list(new_blocks) if resumed else blocks + list(new_blocks)
            if computed + so.num_scheduled_tokens.get(rid, 0) >= len(toks) and rid in self._prefill:
                self._pending_saves.append(StoreSave(rid, toks, blocks))
                del self._prefill[rid]
            elif rid in self._prefill:
                self._prefill[rid] = (toks, blocks)
        for nr in so.scheduled_new_reqs:
            prompt = list(nr.prompt_token_ids or [])
            if len(prompt) >= self._block_size * self._bpc:
                self._prefill[nr.req_id] = (prompt, [])
                step(nr.req_id, prompt, nr.block_ids[0], nr.num_computed_tokens)
        cached = so.scheduled_cached_reqs
        resumed = getattr(cached, "resumed_req_ids", set()) or set()
        for i, rid in enumerate(cached.req_ids):
            if rid in self._prefill:
                nb = cached.new_block_ids[i]
                step(rid, None, nb[0] if nb is not None else [], cached.num_computed_tokens[i], rid in resumed)

    def request_finished(self, request, block_ids):
        self._prefill.pop(request.request_id, None)
        return False, None

    # ------------------------------------------------------------ worker
    def register_kv_caches(self, kv_caches: dict) -> None:
        named = sorted(((layer_index(n, i), t) for i, (n, t) in enumerate(kv_caches.items())
                        if isinstance(t, torch.Tensor) and t.numel() > 0), key=lambda x: x[0])
        if not named:
            raise ValueError("no paged KV caches to register")
        self._layers = [t for _, t in named]
        t = self._layers[0]
        heads, head_size = (t.shape[3], t.shape[4])
        self._store = self._make_store(self._tp_rank, t.device, (self._device_bytes, self._host_bytes),
                                       self._compression, heads, head_size, len(self._layers))

    def start_load_kv(self, forward_context, **kwargs) -> None:
        meta = self._get_connector_metadata()
        if not isinstance(meta, StoreConnectorMetadata) or self._store is None:
            return
        for ld in meta.loads:
            got = self._store.load(ld.token_ids, self._layers, ld.block_ids, num_tokens=ld.num_tokens,
                                   first_block=ld.first_block)
            self.stats["loaded_tokens"] += got
            if got < ld.num_tokens:
                # chunks gone since the lookup: vLLM recomputes these blocks
                first_missing = got // self._block_size
                last = -(-ld.num_tokens // self._block_size)
                self._load_errors.update(ld.block_ids[max(first_missing, ld.first_block):last])
                self._errors_total += 1
                log.warning("store: request %s loaded %d of %d prefix tokens", ld.request_id, got, ld.num_tokens)

    def wait_for_layer_load(self, layer_name: str) -> None:
        return

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata, **kwargs) -> None:
        return

    def wait_for_save(self) -> None:
        """After the forward: store the chunks of the prompts it completed
        (gathered on the forward's stream, so they follow its KV writes)."""
        if not self.has_connector_metadata():
            return
        meta = self._get_connector_metadata()
        if not isinstance(meta, StoreConnectorMetadata) or self._store is None:
            return
        if meta.saves and self._layers[0].is_cuda:
            # the store's background writer copies values on its own stream
            torch.cuda.current_stream(self._layers[0].device).synchronize()
        for sv in meta.saves:
            self.stats["saved_chunks"] += self._store.save(sv.token_ids, self._layers, sv.block_ids)
        if meta.saves and self._layers[0].is_cuda:
            torch.cuda.current_stream(self._layers[0].device).synchronize()

    def get_finished(self, finished_req_ids: set):
        return None, None

    def get_kv_connector_stats(self):
        """This interval's store telemetry, then reset."""
        cur = {"loaded_tokens": self.stats["loaded_tokens"], "saved_chunks": self.stats["saved_chunks"],
               "load_errors": self._errors_total}
        delta = {k: v - self._stats_seen.get(k, 0) for k, v in cur.items()}
        self._stats_seen = cur
        st = StoreStats(data=delta)
        return None if st.is_empty() else st

    @classmethod
    def build_kv_connector_stats(cls, data=None):
        return StoreStats(data=dict(data or {}))

    def get_block_ids_with_load_errors(self) -> set:
        out, self._load_errors = self._load_errors, set()
        return out

    def shutdown(self) -> None:
        for st in (self._store, self._lookup_store):
            if st is not None:
                st.pool.flush()
                st.pool.close()
        self._store = self._lookup_store = None

    @classmethod
    def get_required_kvcache_layout(cls, vllm_config) -> Optional[str]:
        if vllm_config.model_config is None or vllm_config.model_config.use_mla:
            return None
        return "NHD"
