"""Configurable transform stage (kvserve_v1/compression/transformer/kvserve_transformer.py)."""
from __future__ import annotations

import torch

from ..components import Transformer

_KINDS = ("hadamard", "dct", "haar")


class KVServeTransformer(Transformer):
    def __init__(self, **kwargs):
        self.transform_type = None
        self.seed = None
        self.transformer = None
        self.update_params(**kwargs)

    def validate(self) -> None:
        if self.transform_type not in _KINDS:
            raise ValueError(f"Invalid transform type: {self.transform_type}")
        if type(self.seed) is not int:
            raise ValueError("seed must be an integer")

    def update_params(self, **kwargs) -> None:
        kind = kwargs.get("transform_type", self.transform_type or "hadamard")
        seed = kwargs.get("seed", self.seed if self.seed is not None else 0x3333)
        if kind not in _KINDS or type(seed) is not int:
            raise ValueError("expected hadamard/dct/haar and an integer seed")
        if (kind, seed) == (self.transform_type, self.seed):
            return
        if kind == "hadamard":
            from .hadamard import HadamardTransform
            impl = HadamardTransform(seed)
        else:
            from .orthogonal import OrthogonalTransform
            impl = OrthogonalTransform(kind, seed)
        self.transform_type, self.seed, self.transformer = kind, seed, impl

    def transform(self, layer_id: int, tensor: torch.Tensor, **kwargs) -> torch.Tensor:
        if self.transform_type != "hadamard":
            return self.transformer.transform(layer_id, tensor)
        return torch.stack([self.transformer.transform(layer_id, tensor[0]),
                            self.transformer.transform(layer_id, tensor[1])])

    def inverse(self, layer_id: int, tensor: torch.Tensor, **kwargs) -> torch.Tensor:
        if self.transform_type != "hadamard":
            return self.transformer.inverse(layer_id, tensor)
        return torch.stack([self.transformer.inverse(layer_id, tensor[0]),
                            self.transformer.inverse(layer_id, tensor[1])])
