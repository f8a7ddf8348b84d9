"""Chunked lossless byte codec: tuple shuffle -> bit shuffle -> repeated-zero
elimination ("TUPL8_1 BIT_8 RZE_2" in LC-framework notation; method of
Burtscher et al., LC: a framework for lossless compression).  This is this
project's own implementation and container format; it is used for profiles
whose codec is ``"lc"`` and, because nvCOMP's ANS format is closed, also for
``"nvcomp"`` profiles (under the distinct codec id ``kvs-rze-v1``).

Per chunk of ``CHUNK`` bytes (the last may be shorter, padded to 16 bytes):
  1. tuple shuffle: the chunk as [n/8, 8] bytes is transposed to [8, n/8];
  2. bit shuffle: the n bytes become 8 bit planes (plane b = bit b of every
     byte, LSB-first), n/8 bytes each;
  3. RZE_2: 16-bit words; a bitmap (1 bit per word, LSB-first) marks the
     non-zero words, followed by the non-zero words in order.
A chunk whose coded size is not smaller than its input is stored raw.

Container (little endian): ``b"KVLZ"``, u32 version=1, u64 original bytes,
u32 chunk bytes, u32 chunk count, then one u32 per chunk (coded size, bit 31 =
raw), then the chunks back to back, each starting on a 4-byte boundary.
"""
from __future__ import annotations

import os

import struct
from typing import Any

import numpy as np
import torch

MAGIC = b"KVLZ"
VERSION = 1
CHUNK = 16384
_HDR = struct.Struct("<4sIQII")
RAW_FLAG = 1 << 31


def _pad16(n: int) -> int:
    return (n + 15) // 16 * 16


def shuffle_chunk(data: np.ndarray) -> np.ndarray:
    n = data.size
    tup = data.reshape(n // 8, 8).T.reshape(-1)                  # tuple shuffle
    bits = np.unpackbits(tup, bitorder="little").reshape(n, 8)   # [byte, bit]
    planes = np.packbits(bits.T.reshape(-1), bitorder="little")  # 8 planes of n bits
    return planes


def unshuffle_chunk(planes: np.ndarray, n: int) -> np.ndarray:
    bits = np.unpackbits(planes, bitorder="little").reshape(8, n).T
    tup = np.packbits(bits.reshape(-1), bitorder="little")
    return tup.reshape(8, n // 8).T.reshape(-1)


def rze_encode(planes: np.ndarray) -> bytes:
    words = planes.view("<u2")
    nz = words != 0
    bitmap = np.packbits(nz, bitorder="little")
    return bitmap.tobytes() + words[nz].tobytes()


def rze_decode(buf: bytes, n_bytes: int) -> np.ndarray:
    n_words = n_bytes // 2
    bm_bytes = (n_words + 7) // 8
    nz = np.unpackbits(np.frombuffer(buf[:bm_bytes], dtype=np.uint8), bitorder="little")[:n_words].astype(bool)
    words = np.zeros(n_words, dtype="<u2")
    cnt = int(nz.sum())
    words[nz] = np.frombuffer(buf[bm_bytes:bm_bytes + 2 * cnt], dtype="<u2")
    return words.view(np.uint8)


def encode_bytes(data: np.ndarray, chunk: int = CHUNK) -> bytes:
    data = np.ascontiguousarray(data, dtype=np.uint8).reshape(-1)
    total = data.size
    nchunks = (total + chunk - 1) // chunk
    sizes, blobs = [], []
    for c in range(nchunks):
        part = data[c * chunk:(c + 1) * chunk]
        n = _pad16(part.size)
        buf = np.zeros(n, dtype=np.uint8)
        buf[:part.size] = part
        coded = rze_encode(shuffle_chunk(buf))
        if len(coded) >= part.size:
            sizes.append(part.size | RAW_FLAG)
            blobs.append(part.tobytes())
        else:
            sizes.append(len(coded))
            blobs.append(coded)
    out = bytearray(_HDR.pack(MAGIC, VERSION, total, chunk, nchunks))
    out += np.asarray(sizes, dtype="<u4").tobytes()
    for b in blobs:
        out += b
        out += b"\0" * ((-len(b)) % 4)
    return bytes(out)


def decode_bytes(buf: bytes) -> np.ndarray:
    magic, ver, total, chunk, nchunks = _HDR.unpack_from(buf, 0)
    if magic != MAGIC or ver != VERSION:
        raise ValueError("not a kvs-rze-v1 payload")
    sizes = np.frombuffer(buf, dtype="<u4", count=nchunks, offset=_HDR.size)
    pos = _HDR.size + 4 * nchunks
    out = np.empty(total, dtype=np.uint8)
    for c in range(nchunks):
        size = int(sizes[c])
        clen = min(chunk, total - c * chunk)
        if size & RAW_FLAG:
            n = size & ~RAW_FLAG
            out[c * chunk:c * chunk + n] = np.frombuffer(buf, dtype=np.uint8, count=n, offset=pos)
            pos += n + ((-n) % 4)
            continue
        n = _pad16(clen)
        planes = rze_decode(buf[pos:pos + size], n)
        out[c * chunk:c * chunk + clen] = unshuffle_chunk(planes, n)[:clen]
        pos += size + ((-size) % 4)
    return out


class LosslessCodec:
    """Tuple/bit-shuffle + zero-run-elimination codec over any tensor's bytes."""

    codec_id = "kvs-rze-v1"

    def __init__(self, **kwargs: Any) -> None:
        self.chunk = int(kwargs.get("chunk_bytes", CHUNK))
        # KVSERVE_LC_ALGORITHM is the reference's environment default for the
        # chain; KVSERVE_LC_META_PATH (its generated LC runtime) has no role here
        self.algorithm = kwargs.get("lc_algorithm") or os.environ.get("KVSERVE_LC_ALGORITHM") or "TUPL8_1 BIT_8 RZE_2"
        if self.algorithm == self.codec_id:   # the container name selects its one chain
            self.algorithm = "TUPL8_1 BIT_8 RZE_2"
        if self.algorithm not in ("TUPL8_1 BIT_8 RZE_2",):
            raise ValueError(f"unsupported lossless chain {self.algorithm!r}")

    def update_params(self, **kwargs: Any) -> None:
        if "lc_algorithm" in kwargs and kwargs["lc_algorithm"] != self.algorithm:
            self.__init__(**kwargs)

    def encode(self, tensor: torch.Tensor, **kwargs: Any) -> torch.Tensor:
        raw = tensor.contiguous().view(-1).view(torch.uint8)
        if raw.is_cuda:
            from ...ops.lossless import gpu_encode
            return gpu_encode(raw, self.chunk)
        return torch.frombuffer(bytearray(encode_bytes(raw.numpy(), self.chunk)), dtype=torch.uint8)

    def decode(self, compressed: torch.Tensor, original_dtype: str, original_shape: list, device: str,
               **kwargs: Any) -> torch.Tensor:
        dtype = getattr(torch, str(original_dtype).replace("torch.", ""))
        if compressed.is_cuda:
            from ...ops.lossless import gpu_decode
            flat = gpu_decode(compressed)
        else:
            flat = torch.from_numpy(decode_bytes(compressed.numpy().tobytes()))
        return flat.view(dtype).view(*original_shape)
