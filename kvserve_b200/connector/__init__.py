"""vLLM V1 connector entries (loaded lazily so that importing the package
does not import vLLM): the push connector over the credit transport, the
pull connector over the chunked session protocol, and the prefix-store
connector."""

_MODULES = {
    "CompressedKVConnector": "compressed_kv_connector",
    "CompressedKVConnectorMetadata": "compressed_kv_connector",
    "SessionKVConnector": "session_kv_connector",
    "SessionConnectorMetadata": "session_kv_connector",
    "StoreKVConnector": "store_kv_connector",
    "StoreConnectorMetadata": "store_kv_connector",
}


def __getattr__(name):
    mod = _MODULES.get(name)
    if mod is None:
        raise AttributeError(name)
    import importlib
    return getattr(importlib.import_module(f"{__name__}.{mod}"), name)
