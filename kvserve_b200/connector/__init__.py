"""vLLM V1 connector entry (loaded lazily so that importing the package does
not import vLLM)."""


def __getattr__(name):
    if name in ("CompressedKVConnector", "CompressedKVConnectorMetadata"):
        from . import compressed_kv_connector as m
        return getattr(m, name)
    raise AttributeError(name)
