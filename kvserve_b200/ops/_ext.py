"""Loader of the in-tree sm_100a CUDA extension ``kvserve_b200._C``.

There is no fallback: a CUDA op whose extension is missing raises, so a GPU
run can never silently take a PyTorch path instead of the native kernels.
"""
from __future__ import annotations

import functools


class ExtensionMissing(RuntimeError):
    pass


@functools.lru_cache(maxsize=1)
def ext():
    try:
        from kvserve_b200 import _C  # noqa: WPS433
    except ImportError as exc:  # pragma: no cover - depends on the build
        raise ExtensionMissing(
            "kvserve_b200._C is not built; run `python setup.py build_ext --inplace` "
            "in the repository root (sm_100a / B200 only)") from exc
    return _C


def available() -> bool:
    try:
        ext()
        return True
    except ExtensionMissing:
        return False
