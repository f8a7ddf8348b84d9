"""Standalone prefill/decode engine: paged KV cache, layer-streamed KV
hand-off and the PD request loop (the entry points run without vLLM)."""


def __getattr__(name):
    if name in ("PDEngine", "GenerateResult", "RequestTiming"):
        from . import pd
        return getattr(pd, name)
    if name in ("TransferProfile", "KVTransfer"):
        from . import transfer
        return getattr(transfer, name)
    if name == "PagedKVCache":
        from .kv_cache import PagedKVCache
        return PagedKVCache
    raise AttributeError(name)


__all__ = ["PDEngine", "GenerateResult", "RequestTiming", "TransferProfile", "KVTransfer", "PagedKVCache"]
