"""The reference arm of ``bench.py``: the unmodified reference (installed in
``baseline/_ref``) driven through its own public API.

The reference is a vLLM V1 KV connector; its serving path needs two vLLM
engines (producer and consumer) and a model directory.  When that path can
not be brought up on this machine the arm reports why in one line.
"""
from __future__ import annotations

import os

REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                       "baseline", "_ref")


def unavailable_reason() -> str:
    if not os.path.isdir(os.path.join(REF_DIR, "kvserve_v1")):
        return "reference not installed in baseline/_ref (pip install --target baseline/_ref failed)"
    return ("reference serving arm not wired yet: it needs two vLLM V1 engines with the reference "
            "CompressedKVConnector on a dummy-weight Llama-3.1-8B config")
