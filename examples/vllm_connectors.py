"""KV-transfer configurations for vLLM V1 with this framework's connectors.

Three deployments, one helper each (pass the result as
``LLM(..., kv_transfer_config=...)`` or to ``vllm serve`` as JSON):

* push (:func:`push_config`): the prefill engine compresses each request's
  KV after its forward and sends it over the credit transport; the router
  gives both engines the same ``transfer_id`` (:func:`push_params`);
* pull (:func:`pull_config`): the decode engine pulls the prompt KV chunk by
  chunk through the session protocol; the router sends the request to the
  prefill engine with :func:`pull_prefill_params` and forwards the prefill
  output's ``kv_transfer_params`` to the decode engine unchanged;
* prefix store (:func:`store_config`): every engine of a node shares stored
  prompt KV through a directory (``kv_role="kv_both"``).
"""
from __future__ import annotations

from typing import Any, Optional

PUSH_MODULE = "kvserve_b200.connector.compressed_kv_connector"
PULL_MODULE = "kvserve_b200.connector.session_kv_connector"
STORE_MODULE = "kvserve_b200.connector.store_kv_connector"

# the runtime's K4/V4 profile for the pull connector (runtime keys)
RUNTIME_K4V4 = {"enable-compression-pipeline": True, "pipeline": ["transformer", "quantizer"],
                "high_key_num_levels": 16, "low_key_num_levels": 16, "high_value_num_levels": 16,
                "low_value_num_levels": 16, "split_type": "head", "hybrid_ratio": 0.0,
                "logical_blocks_per_chunk": 16}


def push_config(role: str, decode_host: str = "127.0.0.1", base_port: int = 25010,
                compression: Any = "default", data_plane: str = "nccl"):
    """``role``: ``"kv_producer"`` (prefill) or ``"kv_consumer"`` (decode);
    ``compression``: None, ``"default"``, a profile dict (e.g. a file of
    ``configs/compression``) or a controller spec; ``data_plane``: ``nccl``,
    ``ipc`` (CUDA IPC, one node) or ``gloo``."""
    from vllm.config import KVTransferConfig
    if role not in ("kv_producer", "kv_consumer"):
        raise ValueError(f"role must be kv_producer or kv_consumer, got {role!r}")
    return KVTransferConfig(kv_connector="CompressedKVConnector", kv_connector_module_path=PUSH_MODULE,
                            kv_role=role, kv_rank=0 if role == "kv_producer" else 1, kv_parallel_size=2,
                            kv_ip=decode_host, kv_port=base_port,
                            kv_connector_extra_config={"compression": compression, "data_plane": data_plane})


def push_params(transfer_id: str, max_tokens: int = 32, **sampling):
    """Sampling parameters carrying the shared ``transfer_id``."""
    from vllm import SamplingParams
    return SamplingParams(max_tokens=max_tokens, extra_args={"kv_transfer_params": {"transfer_id": transfer_id}},
                          **sampling)


def pull_config(role: str, prefill_host: str = "127.0.0.1", session_port: int = 26100,
                compression: Optional[dict] = None, prefill_tp: Optional[int] = None,
                decode_tp: Optional[int] = None, inline_payloads: bool = False,
                bootstrap_url: Optional[str] = None, engine_id: Optional[str] = None):
    """The pull connector; ``compression`` uses the runtime's keys
    (default :data:`RUNTIME_K4V4`); give both TP sizes when they differ;
    ``inline_payloads`` for engines on different nodes; ``bootstrap_url``
    (``python -m kvserve_b200.session.bootstrap``) lets decode workers find
    prefill ranks by ``engine_id`` instead of host and port."""
    from vllm.config import KVTransferConfig
    extra: dict = {"session_port": session_port, "compression": compression or RUNTIME_K4V4,
                   "inline_payloads": inline_payloads}
    if prefill_tp is not None:
        extra["prefill_tp_size"] = prefill_tp
    if decode_tp is not None:
        extra["decode_tp_size"] = decode_tp
    if bootstrap_url:
        extra["bootstrap_url"] = bootstrap_url
    if engine_id:
        extra["engine_id"] = engine_id
    return KVTransferConfig(kv_connector="SessionKVConnector", kv_connector_module_path=PULL_MODULE, kv_role=role,
                            kv_ip=prefill_host, kv_connector_extra_config=extra)


def pull_prefill_params(transfer_id: str, **sampling):
    """The prefill request of the pull deployment (one token; the KV stays
    with the prefill engine until the decode engine has pulled it)."""
    from vllm import SamplingParams
    return SamplingParams(max_tokens=1, extra_args={"kv_transfer_params": {"do_remote_decode": True,
                                                                           "transfer_id": transfer_id}},
                          **sampling)


def pull_decode_params(prefill_output_params: dict, max_tokens: int = 32, **sampling):
    """The decode request: the prefill output's ``kv_transfer_params`` as is."""
    from vllm import SamplingParams
    return SamplingParams(max_tokens=max_tokens, extra_args={"kv_transfer_params": dict(prefill_output_params)},
                          **sampling)


def store_config(store_dir: str, disk_bytes: Optional[int] = None, compression: Any = None,
                 blocks_per_chunk: int = 16):
    """The prefix-store connector for every engine of a node."""
    from vllm.config import KVTransferConfig
    store: dict = {"dir": store_dir, "blocks_per_chunk": blocks_per_chunk}
    if disk_bytes:
        store["disk_bytes"] = int(disk_bytes)
    return KVTransferConfig(kv_connector="StoreKVConnector", kv_connector_module_path=STORE_MODULE,
                            kv_role="kv_both", kv_connector_extra_config={"store": store,
                                                                          "compression": compression})
