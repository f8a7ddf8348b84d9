"""Random-sign Walsh-Hadamard transform of KV heads.

Behaviour of kvserve_v1/compression/transformer/hadamard_func.py:11-231:
``y = FWHT(sign * x) / sqrt(n)`` over descending power-of-two chunks of the
head dimension (96 -> 64 + 32), computed in fp32 with one rounding to the
input dtype; the inverse is ``sign * FWHT(y) / sqrt(n)``.  Signs are the
seeded Rademacher vectors of :mod:`kvserve_b200.compression.heads`.

CUDA tensors go through the ``fwht_rows`` sm_100a kernel; CPU tensors use an
fp32 matrix product with the Sylvester Hadamard matrix (same maths).
"""
from __future__ import annotations

import math
from functools import lru_cache

import torch

from ..heads import rademacher_signs


def pow2_chunks(dim: int) -> list[int]:
    out, rem = [], dim
    while rem > 0:
        c = 1 << (rem.bit_length() - 1)
        out.append(c)
        rem -= c
    return out


@lru_cache(maxsize=16)
def _hadamard_cpu(n: int) -> torch.Tensor:
    from ...ops.kv_codec import hadamard_matrix
    return hadamard_matrix(n) / math.sqrt(n)


def fwht_cpu(x: torch.Tensor) -> torch.Tensor:
    """Normalised chunked FWHT of the last dim, fp32 result."""
    xf = x.to(torch.float32)
    outs, start = [], 0
    for c in pow2_chunks(x.shape[-1]):
        outs.append(xf[..., start:start + c] @ _hadamard_cpu(c))
        start += c
    return torch.cat(outs, dim=-1)


class HadamardTransform:
    def __init__(self, base_seed: int = 0xC0FEBABE):
        self.base_seed = int(base_seed)
        self._signs: dict = {}

    def signs(self, layer_id: int, num_heads: int, head_dim: int, device, dtype=torch.float32) -> torch.Tensor:
        key = (layer_id, num_heads, head_dim, str(device), dtype)
        s = self._signs.get(key)
        if s is None:
            s = rademacher_signs(self.base_seed, layer_id, num_heads, head_dim).to(device=device, dtype=dtype)
            self._signs[key] = s
        return s

    def _apply(self, layer_id: int, tensor: torch.Tensor, inverse: bool) -> torch.Tensor:
        if tensor.dim() != 4:
            raise ValueError(f"expected [num_blocks, block_size, num_heads, head_dim], got {tuple(tensor.shape)}")
        heads, dim = tensor.shape[-2], tensor.shape[-1]
        if tensor.is_cuda and tensor.dtype == torch.bfloat16:
            from ...ops import ext
            src = tensor.contiguous()
            out = torch.empty_like(src)
            signs = self.signs(layer_id, heads, dim, tensor.device).contiguous()
            ext().fwht_rows(src.view(-1, dim), out.view(-1, dim), signs, inverse)
            return out
        signs = self.signs(layer_id, heads, dim, "cpu").to(tensor.device)
        xf = tensor.to(torch.float32)
        if not inverse:
            y = fwht_cpu(xf * signs)
        else:
            y = fwht_cpu(xf) * signs
        return y.to(tensor.dtype)

    def transform(self, layer_id: int, tensor: torch.Tensor, **kwargs) -> torch.Tensor:
        return self._apply(layer_id, tensor, False)

    def inverse(self, layer_id: int, tensor: torch.Tensor, **kwargs) -> torch.Tensor:
        return self._apply(layer_id, tensor, True)
