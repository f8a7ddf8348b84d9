"""Seeded dense orthogonal rotations of the head dimension: signed DCT-II and
Haar-random (behaviour of kvserve_v1/compression/transformer/orthogonal.py).

* DCT-II: orthonormal ``B[n, k] = sqrt(2/D) cos(pi/D (n + 1/2) k)`` (column 0
  divided by sqrt 2), with per-(layer, head) Rademacher signs seeded
  ``seed ^ (layer << 16) ^ head``.
* Haar: Q of the QR factorisation of a seeded Gaussian matrix
  (``seed ^ (layer << 16)``), columns sign-fixed by ``sign(diag R)``; no signs.

Forward ``y = (x * sign) @ B``, inverse ``x = (y @ B^T) * sign``.  The fp32
basis is split into bf16 ``hi + lo`` parts; on CUDA both products run on the
tcgen05 GEMM (``x @ hi`` accumulated onto ``x @ lo``), on CPU in fp32.
"""
from __future__ import annotations

import math
from functools import lru_cache

import torch


@lru_cache(maxsize=128)
def orthogonal_basis(kind: str, dim: int, seed: int, layer_id: int) -> torch.Tensor:
    if kind == "dct":
        idx = torch.arange(dim, dtype=torch.float64)
        base = torch.cos(math.pi / dim * (idx[:, None] + 0.5) * idx[None, :]) * math.sqrt(2.0 / dim)
        base[:, 0] /= math.sqrt(2.0)
        return base.float().contiguous()
    if kind == "haar":
        g = torch.Generator(device="cpu")
        g.manual_seed((seed ^ (layer_id << 16)) & ((1 << 63) - 1))
        q, r = torch.linalg.qr(torch.randn(dim, dim, generator=g, dtype=torch.float64))
        q = q * torch.where(r.diagonal() < 0, -1.0, 1.0)[None, :]
        return q.float().contiguous()
    raise ValueError(f"unknown orthogonal transform {kind!r}")


@lru_cache(maxsize=256)
def orthogonal_signs(kind: str, dim: int, heads: int, seed: int, layer_id: int) -> torch.Tensor:
    if kind == "haar":
        return torch.ones((heads, dim), dtype=torch.float32)
    g = torch.Generator(device="cpu")
    out = []
    for h in range(heads):
        g.manual_seed((seed ^ (layer_id << 16) ^ h) & ((1 << 63) - 1))
        out.append(torch.randint(2, (dim,), generator=g) * 2 - 1)
    return torch.stack(out).float()


class OrthogonalTransform:
    """Rotation of ``[2, blocks, tokens, heads, dim]`` KV (layout preserved)."""

    def __init__(self, kind: str = "dct", seed: int = 0x3333):
        if kind not in ("dct", "haar") or type(seed) is not int:
            raise ValueError("expected dct/haar and an integer seed")
        self.kind, self.seed = kind, seed
        self._dev: dict = {}

    def _weights(self, layer_id: int, heads: int, dim: int, device):
        key = (layer_id, heads, dim, str(device))
        w = self._dev.get(key)
        if w is None:
            base = orthogonal_basis(self.kind, dim, self.seed, layer_id)
            hi = base.to(torch.bfloat16)
            lo = (base - hi.float()).to(torch.bfloat16)
            signs = orthogonal_signs(self.kind, dim, heads, self.seed, layer_id)
            # GEMM operands are [N, K]: forward uses B^T, inverse uses B.
            w = {
                "fwd_hi": hi.t().contiguous().to(device), "fwd_lo": lo.t().contiguous().to(device),
                "inv_hi": hi.contiguous().to(device), "inv_lo": lo.contiguous().to(device),
                "base": base.to(device), "signs": signs.to(device),
            }
            self._dev[key] = w
        return w

    def _apply(self, layer_id: int, tensor: torch.Tensor, inverse: bool) -> torch.Tensor:
        if tensor.ndim != 5 or tensor.shape[0] != 2:
            raise ValueError("expected KV [2, blocks, tokens, heads, dim]")
        heads, dim = tensor.shape[-2], tensor.shape[-1]
        if not 1 <= dim <= 512:
            raise ValueError("orthogonal transforms support head dimensions 1-512")
        w = self._weights(layer_id, heads, dim, tensor.device)
        signs = w["signs"].to(torch.float32)
        if tensor.is_cuda and tensor.dtype == torch.bfloat16 and dim % 8 == 0:
            from ... import ops
            x = tensor.contiguous()
            if not inverse and self.kind == "dct":
                x = (x.float() * signs).to(torch.bfloat16)
            rows = x.reshape(-1, dim)
            hi, lo = (w["inv_hi"], w["inv_lo"]) if inverse else (w["fwd_hi"], w["fwd_lo"])
            y = ops.gemm(rows, hi, residual=ops.gemm(rows, lo)).view(tensor.shape)
            if inverse and self.kind == "dct":
                y = (y.float() * signs).to(torch.bfloat16)
            return y
        xf = tensor.to(torch.float32)
        base = w["base"].to(torch.float32)
        if not inverse:
            y = (xf * signs) @ base
        else:
            y = (xf @ base.t()) * signs
        return y.to(tensor.dtype)

    def transform(self, layer_id: int, tensor: torch.Tensor, **kwargs) -> torch.Tensor:
        return self._apply(layer_id, tensor, False)

    def inverse(self, layer_id: int, tensor: torch.Tensor, **kwargs) -> torch.Tensor:
        return self._apply(layer_id, tensor, True)
