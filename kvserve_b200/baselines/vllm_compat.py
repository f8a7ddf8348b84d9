"""vLLM-API adapter under which the reference's consumer runs on vLLM 0.22.

The reference connector was written against an older vLLM V1 in which every
attention layer kept one KV cache per virtual engine (``layer.kv_cache`` a
list) and the forward context named the current one (``virtual_engine``).
Its consumer injects received KV with
``layer.kv_cache[forward_context.virtual_engine]``
(kvserve_v1/connector/compressed_kv_connector.py:346-355).  vLLM 0.22 keeps a
single cache tensor per layer and has no ``virtual_engine`` field, so the
stock consumer raises ``AttributeError`` on its first request.

This module changes nothing in the reference.  It is a vLLM general plugin
(entry point group ``vllm.general_plugins``, loaded by vLLM in the engine
core and every worker process) that wraps vLLM's own call site of
``start_load_kv``: the connector receives a read-only view of the forward
context in the older shape — ``virtual_engine == 0`` and each layer's
``kv_cache`` as a one-element list holding the real cache tensor.  Every
other attribute reads through to vLLM's objects, and the tensor handed out
is vLLM's own cache, so the reference's inject writes the real KV cache.

:func:`install_entry_point` writes the plugin's distribution metadata into a
directory; put that directory on ``PYTHONPATH`` (and name the plugin in
``VLLM_PLUGINS``) for the reference processes only.
"""
from __future__ import annotations

import os
from collections.abc import Mapping

PLUGIN_NAME = "kvs_ref_vllm_compat"


class _LayerView:
    """An attention layer whose ``kv_cache`` is the per-virtual-engine list."""

    __slots__ = ("_layer",)

    def __init__(self, layer):
        object.__setattr__(self, "_layer", layer)

    @property
    def kv_cache(self):
        kv = getattr(self._layer, "kv_cache", None)
        if kv is None or isinstance(kv, (list, tuple)):
            return kv
        return [kv]

    def __getattr__(self, name):
        return getattr(self._layer, name)


class _LayersView(Mapping):
    def __init__(self, layers):
        self._layers = layers

    def __getitem__(self, name):
        return _LayerView(self._layers[name])

    def __iter__(self):
        return iter(self._layers)

    def __len__(self):
        return len(self._layers)


class ForwardContextView:
    """The forward context as the older vLLM exposed it to connectors."""

    virtual_engine = 0

    def __init__(self, ctx):
        object.__setattr__(self, "_ctx", ctx)

    @property
    def no_compile_layers(self):
        return _LayersView(self._ctx.no_compile_layers)

    def __getattr__(self, name):
        return getattr(self._ctx, name)


def _wrap_module(mod) -> bool:
    """Make ``mod.get_forward_context`` (used there only to call
    ``start_load_kv``) return the view."""
    orig = getattr(mod, "get_forward_context", None)
    if orig is None or getattr(orig, "_kvs_compat", False):
        return False

    def get_forward_context_view():
        return ForwardContextView(orig())

    get_forward_context_view._kvs_compat = True
    mod.get_forward_context = get_forward_context_view
    return True


def register() -> None:
    """vLLM general-plugin hook (runs in every vLLM process)."""
    import importlib
    for name in ("vllm.v1.worker.kv_connector_model_runner_mixin", "vllm.v1.worker.gpu.kv_connector"):
        try:
            _wrap_module(importlib.import_module(name))
        except ImportError:
            continue


def install_entry_point(directory: str) -> str:
    """Write ``<directory>/kvs_ref_vllm_compat-0.dist-info`` declaring
    :func:`register` as a vLLM general plugin; returns ``directory``."""
    info = os.path.join(directory, f"{PLUGIN_NAME}-0.dist-info")
    os.makedirs(info, exist_ok=True)
    with open(os.path.join(info, "METADATA"), "w") as f:
        f.write(f"Metadata-Version: 2.1\nName: {PLUGIN_NAME}\nVersion: 0\n")
    with open(os.path.join(info, "entry_points.txt"), "w") as f:
        f.write(f"[vllm.general_plugins]\n{PLUGIN_NAME} = kvserve_b200.baselines.vllm_compat:register\n")
    return directory
