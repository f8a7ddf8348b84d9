"""BitPack codec: lossless fixed-width packing of bounded uint8 symbols.

Format (identical to kvserve_v1/compression/codec/bitpack_codec.py:20-69):
16-byte header = magic ``0x0150424B`` (LE u32), ``bits`` (u8), three zero
bytes, symbol count (LE u64); then the symbols in tensor order packed
least-significant-bit first, ``ceil(count * bits / 8)`` bytes.

CUDA tensors use the sm_100a ``bitpack_encode``/``bitpack_decode`` kernels,
which report an out-of-range symbol or a header mismatch through a status
word (raised here as ``ValueError``) instead of a device assert; CPU tensors
use numpy.
"""
from __future__ import annotations

import math
from typing import Any

import numpy as np
import torch

HEADER_BYTES = 16
MAGIC = 0x0150424B


def _width(kwargs: dict, default: int) -> int:
    bits = kwargs.get("bitpack_bits", default)
    if type(bits) is not int or not 1 <= bits <= 8:
        raise ValueError("bitpack_bits must be an integer in [1, 8]")
    return bits


def pack_cpu(sym: np.ndarray, bits: int) -> np.ndarray:
    from ...ops.kv_codec import _pack_bits, bitpack_header
    if sym.size and int(sym.max()) >= (1 << bits):
        raise ValueError("symbol exceeds bitpack_bits")
    return np.frombuffer(bitpack_header(bits, sym.size) + _pack_bits(sym, bits), dtype=np.uint8).copy()


def unpack_cpu(buf: np.ndarray, bits: int, count: int) -> np.ndarray:
    from ...ops.kv_codec import _unpack_bits, bitpack_header
    if bytes(buf[:16].tobytes()) != bitpack_header(bits, count):
        raise ValueError("invalid bitpack header or decode configuration")
    return _unpack_bits(buf[16:].tobytes(), bits, count)


class BitPackCodec:
    def __init__(self, **kwargs: Any) -> None:
        self.bitpack_bits = 8
        self.update_params(**kwargs)

    def update_params(self, **kwargs: Any) -> None:
        self.bitpack_bits = _width(kwargs, self.bitpack_bits)

    @staticmethod
    def _check(t: torch.Tensor) -> None:
        if not isinstance(t, torch.Tensor) or t.dtype != torch.uint8:
            raise TypeError("BitPackCodec requires a torch.uint8 tensor")

    def encode(self, tensor: torch.Tensor, **kwargs: Any) -> torch.Tensor:
        bits = _width(kwargs, self.bitpack_bits)
        self._check(tensor)
        src = tensor.contiguous().view(-1)
        n = src.numel()
        if not tensor.is_cuda:
            return torch.from_numpy(pack_cpu(src.numpy(), bits))
        from ...ops import ext
        out = torch.empty(HEADER_BYTES + (n * bits + 7) // 8, dtype=torch.uint8, device=tensor.device)
        status = torch.zeros(1, dtype=torch.int32, device=tensor.device)
        with torch.cuda.device(tensor.device):
            ext().bitpack_encode(src, out, bits, status)
        if int(status.item()) != 0:
            raise ValueError("symbol exceeds bitpack_bits")
        return out

    def decode(self, compressed: torch.Tensor, original_dtype: str, original_shape: list, device: str,
               **kwargs: Any) -> torch.Tensor:
        bits = _width(kwargs, self.bitpack_bits)
        self._check(compressed)
        if str(original_dtype).replace("torch.", "") != "uint8":
            raise TypeError("BitPackCodec restores uint8 symbols only")
        if any(type(d) is not int or d < 0 for d in original_shape):
            raise ValueError("original_shape must contain nonnegative integers")
        count = math.prod(original_shape)
        if compressed.numel() != HEADER_BYTES + (count * bits + 7) // 8:
            raise ValueError("BitPackCodec payload length does not match shape and bit width")
        if not compressed.is_cuda:
            return torch.from_numpy(unpack_cpu(compressed.numpy(), bits, count)).view(*original_shape)
        from ...ops import ext
        out = torch.empty(original_shape, dtype=torch.uint8, device=compressed.device)
        status = torch.zeros(1, dtype=torch.int32, device=compressed.device)
        with torch.cuda.device(compressed.device):
            ext().bitpack_decode(compressed.contiguous(), out, bits, status)
        if int(status.item()) != 0:
            raise ValueError("invalid bitpack header or decode configuration")
        return out
