"""GPU front-end of the ``kvs-rze-v1`` lossless codec (``csrc/lossless.cu``).
The encoded bytes are identical to the CPU implementation in
``kvserve_b200.compression.codec.lossless``."""
from __future__ import annotations

import struct

import torch

from . import count_launches
from ._ext import ext

CHUNK = 16384
_HDR = struct.Struct("<4sIQII")


def gpu_encode(raw: torch.Tensor, chunk: int = CHUNK) -> torch.Tensor:
    """Encode a contiguous uint8 CUDA tensor; returns a view of the exact size
    (reading the size synchronises with the stream once)."""
    n = raw.numel()
    out = torch.empty(ext().rze_max_encoded_bytes(n, chunk), dtype=torch.uint8, device=raw.device)
    scratch = torch.empty(ext().rze_scratch_bytes(n, chunk), dtype=torch.uint8, device=raw.device)
    total = torch.empty(1, dtype=torch.int64, device=raw.device)
    count_launches(3)
    ext().rze_encode(raw, out, scratch, total, chunk)
    return out[: int(total.item())]


def gpu_decode(payload: torch.Tensor) -> torch.Tensor:
    hdr = bytes(payload[: _HDR.size].cpu().numpy().tobytes())
    magic, ver, total, chunk, nchunks = _HDR.unpack(hdr)
    if magic != b"KVLZ" or ver != 1:
        raise ValueError("not a kvs-rze-v1 payload")
    out = torch.empty(total, dtype=torch.uint8, device=payload.device)
    scratch = torch.empty(8 * nchunks + 32, dtype=torch.uint8, device=payload.device)
    count_launches(2)
    ext().rze_decode(payload.contiguous(), out, scratch, chunk)
    return out
