"""kvserve_b200 — a Blackwell-native (B200, sm_100a) framework for
disaggregated prefill/decode serving with compressed KV transfer.

Public entry points are imported lazily so that ``import kvserve_b200`` stays
cheap and works without a GPU.
"""
from __future__ import annotations

__version__ = "0.1.0"

_LAZY = {
    "CompressedKVConnector": "kvserve_b200.connector.compressed_kv_connector",
    "SessionKVConnector": "kvserve_b200.connector.session_kv_connector",
    "StoreKVConnector": "kvserve_b200.connector.store_kv_connector",
    "KVCompressionAdapter": "kvserve_b200.compression.adapter",
    "CompressionManager": "kvserve_b200.compression.manager",
    "PDEngine": "kvserve_b200.engine.pd",
    "LLM": "kvserve_b200.engine.api",
}


def __getattr__(name):
    mod = _LAZY.get(name)
    if mod is None:
        raise AttributeError(name)
    import importlib
    return getattr(importlib.import_module(mod), name)
