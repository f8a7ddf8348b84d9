"""Transform stage of the modular pipeline, selected by ``transform_type``.

Every transform this stage can run is an entry of a registry: the entry
names the kind, checks the parameters it accepts, and builds the
implementation for a seed.  The stage itself only resolves a parameter set
against the registry and applies the implementation to one layer
``[2, blocks, tokens, heads, dim]`` (K and V halves).  Entries that work on a
single half (the Hadamard path, whose kernels take ``[blocks, tokens, heads,
dim]``) are applied to each half; whole-layer entries receive the layer.

Kinds and parameters match the profiles of
kvserve_v1/compression/transformer/kvserve_transformer.py:7-51 (``hadamard``,
``dct``, ``haar``; an integer ``seed``), plus ``hadamard_bf16``: the same
transform with the reference runtime's numerics (bf16 rounding after every
butterfly stage), which reproduces that runtime's quantisation symbols.  A profile that omits the seed
implies ``DEFAULT_SEED``: it selects the random signs, so both peers (and a
reference peer) must derive the same value.  New kinds are added with
:func:`register_transform`.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Optional

import torch

from ..components import Transformer

DEFAULT_KIND = "hadamard"
DEFAULT_SEED = 0x3333


@dataclass(frozen=True)
class TransformKind:
    """One registered transform: how to build it and how it takes a layer."""
    name: str
    factory: Callable[[int], Any]
    per_half: bool

    def check(self, seed: Any) -> int:
        # bool is an int subclass but never a meaningful seed
        if isinstance(seed, bool) or not isinstance(seed, int):
            raise ValueError(f"transform {self.name!r}: seed must be an integer, got {seed!r}")
        return seed


_REGISTRY: dict[str, TransformKind] = {}


def register_transform(name: str, factory: Callable[[int], Any], per_half: bool = False) -> None:
    """Make ``transform_type=name`` available; ``factory(seed)`` returns an
    object with ``transform(layer_id, x)`` / ``inverse(layer_id, x)``."""
    _REGISTRY[name] = TransformKind(name, factory, per_half)


def registered_transforms() -> tuple[str, ...]:
    return tuple(sorted(_REGISTRY))


def _hadamard(seed: int):
    from .hadamard import HadamardTransform
    return HadamardTransform(seed)


def _hadamard_bf16(seed: int):
    from .hadamard import HadamardTransform
    return HadamardTransform(seed, numerics="bf16-stagewise")


def _rotation(kind: str) -> Callable[[int], Any]:
    def make(seed: int):
        from .orthogonal import OrthogonalTransform
        return OrthogonalTransform(kind, seed)
    return make


register_transform("hadamard", _hadamard, per_half=True)
# the reference runtime's numerics (bf16 rounding after every butterfly stage)
register_transform("hadamard_bf16", _hadamard_bf16, per_half=True)
register_transform("dct", _rotation("dct"))
register_transform("haar", _rotation("haar"))


def resolve(params: dict, current: Optional[tuple[str, int]] = None) -> tuple[TransformKind, int]:
    """Registry entry and seed for ``params``; keys that are absent keep the
    ``current`` setting (or the defaults on first use)."""
    name = params.get("transform_type", current[0] if current else DEFAULT_KIND)
    entry = _REGISTRY.get(name)
    if entry is None:
        raise ValueError(f"unknown transform_type {name!r}; registered: {', '.join(registered_transforms())}")
    seed = entry.check(params.get("seed", current[1] if current else DEFAULT_SEED))
    return entry, seed


class KVServeTransformer(Transformer):
    """Configurable transform stage (``pipeline`` entry ``"transformer"``)."""

    def __init__(self, **params: Any):
        self._entry: Optional[TransformKind] = None
        self._seed: Optional[int] = None
        self._impl: Any = None
        self.update_params(**params)

    @property
    def transform_type(self) -> Optional[str]:
        return self._entry.name if self._entry else None

    @property
    def seed(self) -> Optional[int]:
        return self._seed

    @property
    def transformer(self) -> Any:
        """The implementation object of the selected kind."""
        return self._impl

    def validate(self) -> None:
        resolve({}, (self.transform_type, self._seed) if self._entry else None)

    def update_params(self, **params: Any) -> None:
        current = (self._entry.name, self._seed) if self._entry else None
        entry, seed = resolve(params, current)
        if self._impl is not None and (entry.name, seed) == current:
            return  # signs / bases are cached inside the implementation
        self._entry, self._seed, self._impl = entry, seed, entry.factory(seed)

    def _run(self, op: str, layer_id: int, layer: torch.Tensor) -> torch.Tensor:
        fn = getattr(self._impl, op)
        if not self._entry.per_half:
            return fn(layer_id, layer)
        return torch.stack([fn(layer_id, layer[half]) for half in range(layer.shape[0])])

    def transform(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any) -> torch.Tensor:
        return self._run("transform", layer_id, tensor)

    def inverse(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any) -> torch.Tensor:
        return self._run("inverse", layer_id, tensor)
