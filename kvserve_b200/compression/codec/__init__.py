"""Codec stage: dispatch over the supported lossless codecs
(behaviour of kvserve_v1/compression/codec/kvserve_codec.py).

``codec_type``:
* ``"bitpack"`` — fixed-width BitPack (byte-identical format);
* ``"lc"`` — this project's tuple/bit-shuffle + zero-run codec (LC-style
  ``TUPL8_1 BIT_8 RZE_2`` chain, own container ``kvs-rze-v1``);
* ``"nvcomp"`` — nvCOMP's formats are closed, so these profiles run the same
  lossless codec under the distinct id ``kvs-rze-v1``; payloads are not
  nvCOMP-compatible (the algorithm name is validated and recorded).
"""
from __future__ import annotations

from typing import Any

import torch

from ..components import Codec
from .bitpack import BitPackCodec
from .lossless import LosslessCodec

_NVCOMP_ALGOS = ("ANS", "Bitcomp", "Cascaded", "Deflate", "GDeflate", "LZ4", "Zstd")
_TYPES = ("nvcomp", "lc", "bitpack")


class KVServeCodec(Codec):
    def __init__(self, **kwargs: Any) -> None:
        self.codec_type = kwargs.get("codec_type", "nvcomp")
        self.nvcomp_algorithm = kwargs.get("nvcomp_algorithm", "ANS")
        self.lc_algorithm = kwargs.get("lc_algorithm")
        self._kwargs = dict(kwargs)
        self.codec = None
        self.validate()
        self._build()

    def validate(self) -> None:
        if self.codec_type not in _TYPES:
            raise ValueError(f"Invalid codec type: {self.codec_type}, expected one of: {list(_TYPES)}")
        if self.codec_type == "nvcomp" and self.nvcomp_algorithm not in _NVCOMP_ALGOS:
            raise ValueError(f"Invalid nvcomp's algorithm: {self.nvcomp_algorithm}")

    def _build(self) -> None:
        if self.codec_type == "bitpack":
            self.codec = BitPackCodec(**self._kwargs)
        else:
            kw = dict(self._kwargs)
            kw.setdefault("lc_algorithm", "TUPL8_1 BIT_8 RZE_2")
            if self.codec_type == "lc" and not kw.get("lc_algorithm"):
                kw["lc_algorithm"] = "TUPL8_1 BIT_8 RZE_2"
            if self.codec_type == "nvcomp":
                kw["lc_algorithm"] = "TUPL8_1 BIT_8 RZE_2"
            self.codec = LosslessCodec(**kw)

    @property
    def codec_id(self) -> str:
        return "bitpack-v1" if self.codec_type == "bitpack" else LosslessCodec.codec_id

    def update_params(self, **kwargs: Any) -> None:
        prev = (self.codec_type, self.nvcomp_algorithm, self.lc_algorithm)
        self._kwargs.update(kwargs)
        for k in ("codec_type", "nvcomp_algorithm", "lc_algorithm"):
            if k in kwargs:
                setattr(self, k, kwargs[k])
        self.validate()
        if (self.codec_type, self.nvcomp_algorithm, self.lc_algorithm) != prev or self.codec is None:
            self._build()
        else:
            self.codec.update_params(**kwargs)

    def encode(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any) -> torch.Tensor:
        return self.codec.encode(tensor, **kwargs)

    def decode(self, layer_id: int, tensor: torch.Tensor, original_dtype: str, original_shape: list, device: str,
               **kwargs: Any) -> torch.Tensor:
        return self.codec.decode(tensor, original_dtype, original_shape, device, **kwargs)


__all__ = ["KVServeCodec", "BitPackCodec", "LosslessCodec"]
