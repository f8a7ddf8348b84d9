"""Random-sign Walsh-Hadamard transform of KV heads.

Behaviour of kvserve_v1/compression/transformer/hadamard_func.py:11-231:
``y = FWHT(sign * x) / sqrt(n)`` over descending power-of-two chunks of the
head dimension (96 -> 64 + 32), computed in fp32 with one rounding to the
input dtype; the inverse is ``sign * FWHT(y) / sqrt(n)``.  Signs are the
seeded Rademacher vectors of :mod:`kvserve_b200.compression.heads`.

CUDA tensors go through the ``fwht_rows`` sm_100a kernel; CPU tensors use an
fp32 matrix product with the Sylvester Hadamard matrix (same maths).

``numerics="bf16-stagewise"`` reproduces the reference runtime's symbols
instead (kvserve_v1/compression/runtime/csrc/kvs_compress.cu:119-161 and its
CPU twin, runtime/pipeline.py:307-335): the signed input is rounded to bf16,
every butterfly stage (strides 1, 2, 4, ...) is rounded to bf16, and so is
the final ``1/sqrt(n)`` scale; the inverse runs the same transform and then
multiplies by the signs (rounded).  Power-of-two head sizes only.
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


def fwht_bf16_stagewise(x: torch.Tensor) -> torch.Tensor:
    """Normalised FWHT of the last dim (a power of two) with a bf16 rounding
    after every butterfly stage and after the scale; bf16 result."""
    n = x.shape[-1]
    if n & (n - 1):
        raise ValueError("the stage-wise bf16 FWHT needs a power-of-two size")
    lead = x.shape[:-1]
    y = x.to(torch.bfloat16).to(torch.float32)
    step = 1
    while step < n:
        pairs = y.reshape(*lead, n // (2 * step), 2, step)
        a, b = pairs[..., 0, :], pairs[..., 1, :]
        y = torch.stack((a + b, a - b), dim=-2).to(torch.bfloat16).to(torch.float32)
        step *= 2
    # 1/sqrt(n) evaluated in fp32, as the kernel does
    scale = torch.tensor(1.0, dtype=torch.float32) / torch.sqrt(torch.tensor(float(n), dtype=torch.float32))
    return (y.reshape(x.shape) * scale.to(y.device)).to(torch.bfloat16)


NUMERICS = ("fp32", "bf16-stagewise")


class HadamardTransform:
    def __init__(self, base_seed: int = 0xC0FEBABE, numerics: str = "fp32"):
        if numerics not in NUMERICS:
            raise ValueError(f"numerics must be one of {NUMERICS}, got {numerics!r}")
        self.base_seed = int(base_seed)
        self.numerics = numerics
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
        if self.numerics == "bf16-stagewise":
            signs = self.signs(layer_id, heads, dim, tensor.device, torch.bfloat16)
            if not inverse:
                return fwht_bf16_stagewise(tensor.to(torch.bfloat16) * signs).to(tensor.dtype)
            return (fwht_bf16_stagewise(tensor) * signs).to(tensor.dtype)
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
