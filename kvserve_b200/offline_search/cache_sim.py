"""KV-compression simulators for offline evaluation (role of
kvserve_v1/offline_search/src/cache/{cache_utils,kivi_utils,cachegen_utils,duoattn_utils}.py).

Each simulator maps a KV sample ``[L, 2, B, S, H, D]`` to its reconstruction
and a compression ratio (original bytes / stored bytes, metadata included),
so methods can be compared on the same data with the same evaluators:

* :class:`KVServeSim` — this framework's modular pipeline (any profile).
* :class:`KIVISim` — KIVI-style asymmetric quantisation: keys per channel in
  groups of ``group`` tokens, values per token in groups of ``group``
  channels, the newest ``S mod residual`` tokens kept in 16 bit.
* :class:`CacheGenSim` — CacheGen-style delta coding: tokens in chunks of
  ``chunk``, each token coded as the delta to its chunk's anchor token,
  layer-group dependent bin counts, size estimated as the empirical entropy
  of the symbols (the bound an arithmetic coder approaches) plus anchors.
* :class:`DuoAttentionSim` — streaming heads (the lowest-score fraction)
  keep ``sink`` + ``recent`` tokens, retrieval heads keep everything.

:func:`simulated_cache` wraps any simulator as a Hugging Face
``DynamicCache`` whose prefill update stores the reconstruction, so a model
run sees exactly the degraded KV.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Sequence

import torch


def _bytes(t_elems: int, bits: float) -> float:
    return t_elems * bits / 8.0


def _minmax_qdq(x: torch.Tensor, bits: int, dim: int) -> tuple[torch.Tensor, int]:
    """Asymmetric min/max quantise-dequantise along ``dim`` (groups are the
    other dims); returns the reconstruction and the number of groups."""
    mn = x.amin(dim=dim, keepdim=True)
    mx = x.amax(dim=dim, keepdim=True)
    levels = (1 << bits) - 1
    scale = (mx - mn).clamp_min(1e-6) / levels
    q = ((x - mn) / scale).round().clamp_(0, levels)
    return q * scale + mn, mn.numel()


@dataclass
class KIVISim:
    bits: int = 2
    group: int = 32
    residual: int = 128

    def __call__(self, kv: torch.Tensor) -> tuple[torch.Tensor, float]:
        L, _, B, S, H, D = kv.shape
        x = kv.float()
        out = x.clone()
        qlen = (S // self.residual) * self.residual if self.residual else S
        stored = 0.0
        if qlen:
            k = x[:, 0, :, :qlen]                                  # [L, B, qlen, H, D]
            g = self.group
            kt = k[:, :, : qlen // g * g].reshape(L, B, qlen // g, g, H, D)
            kr, ng_k = _minmax_qdq(kt, self.bits, dim=3)            # per channel over g tokens
            out[:, 0, :, : qlen // g * g] = kr.reshape(L, B, qlen // g * g, H, D)
            v = x[:, 1, :, :qlen]
            vt = v.reshape(L, B, qlen, H, D // g, g)
            vr, ng_v = _minmax_qdq(vt, self.bits, dim=5)            # per token over g channels
            out[:, 1, :, :qlen] = vr.reshape(L, B, qlen, H, D)
            stored += _bytes(2 * L * B * qlen * H * D, self.bits) + 2 * 2 * (ng_k + ng_v)
        stored += 2 * 2 * L * B * (S - qlen) * H * D
        orig = 2 * kv.numel()
        return out.to(kv.dtype), orig / max(1.0, stored)


@dataclass
class CacheGenSim:
    chunk: int = 10
    bins: Sequence[int] = (32, 16, 16)   # per layer third: early, middle, late
    anchor_bits: int = 8

    @staticmethod
    def _entropy_bits(sym: torch.Tensor) -> float:
        _, counts = torch.unique(sym, return_counts=True)
        p = counts.double() / sym.numel()
        return float(-(p * p.log2()).sum()) * sym.numel()

    def __call__(self, kv: torch.Tensor) -> tuple[torch.Tensor, float]:
        L, P, B, S, H, D = kv.shape
        x = kv.float()
        out = torch.empty_like(x)
        bits_total = 0.0
        for l in range(L):
            nb = self.bins[min(len(self.bins) - 1, 3 * l // max(1, L))]
            for p in range(P):
                t = x[l, p]                                          # [B, S, H, D]
                pad = (-S) % self.chunk
                tp = torch.cat([t, t[:, -1:].expand(B, pad, H, D)], 1) if pad else t
                c = tp.reshape(B, -1, self.chunk, H, D)
                anchor = c[:, :, :1]
                # anchors at anchor_bits, per channel over the tensor
                a_rec, _ = _minmax_qdq(anchor, self.anchor_bits, dim=1)
                delta = c - a_rec
                rng = delta.abs().amax(dim=(0, 1, 2), keepdim=True).clamp_min(1e-6)
                step = 2 * rng / nb
                sym = (delta / step).round().clamp_(-(nb // 2), nb // 2)
                rec = a_rec + sym * step
                out[l, p] = rec.reshape(B, -1, H, D)[:, :S]
                bits_total += self._entropy_bits(sym[:, :, 1:]) + anchor.numel() * self.anchor_bits \
                    + 2 * 32 * H * D
        orig = 2 * kv.numel()
        return out.to(kv.dtype), orig / max(1.0, bits_total / 8.0)


@dataclass
class DuoAttentionSim:
    sparsity: float = 0.5
    sink: int = 64
    recent: int = 256
    scores: Optional[torch.Tensor] = None   # [L, H]; lower = streaming head

    def head_mask(self, L: int, H: int) -> torch.Tensor:
        s = self.scores if self.scores is not None else torch.linspace(0, 1, L * H).view(L, H)
        n = round(L * H * self.sparsity)
        mask = torch.zeros(L * H, dtype=torch.bool)
        mask[torch.argsort(s.reshape(-1), stable=True)[:n]] = True
        return mask.view(L, H)                                      # True = streaming

    def __call__(self, kv: torch.Tensor) -> tuple[torch.Tensor, float]:
        L, _, B, S, H, D = kv.shape
        keep = torch.zeros(S, dtype=torch.bool)
        keep[: self.sink] = True
        keep[max(0, S - self.recent):] = True
        out = kv.clone()
        mask = self.head_mask(L, H)
        for l in range(L):
            for h in range(H):
                if mask[l, h]:
                    out[l, :, :, ~keep, h] = 0
        kept_tokens = int(keep.sum())
        stored = (mask.sum() * kept_tokens + (~mask).sum() * S).item()
        return out, (L * H * S) / max(1, stored)


class KVServeSim:
    """This framework's modular pipeline on the sample (any compression
    profile accepted by :class:`~kvserve_b200.compression.adapter.KVCompressionAdapter`)."""

    def __init__(self, config: dict, num_kv_heads: int, head_size: int, num_layers: Optional[int] = None):
        from ..compression.adapter import KVCompressionAdapter
        self.adapter = KVCompressionAdapter(config, num_kv_heads, head_size, num_layers=num_layers)

    def __call__(self, kv: torch.Tensor) -> tuple[torch.Tensor, float]:
        c = self.adapter.compress(kv, "sim")
        if c is None:
            return kv, 1.0
        return self.adapter.decompress(c).to(kv.dtype), c.original_size / max(1, c.compressed_size)


def simulated_cache(sim, num_layers: int):
    """A ``transformers`` ``DynamicCache`` that replaces each layer's prefill
    K/V (``[B, H, S, D]``) by ``sim``'s reconstruction before storing it.
    The per-layer ratios are kept in ``cache.ratios``."""
    from transformers import DynamicCache

    class _SimCache(DynamicCache):
        def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
            if key_states.shape[-2] > 1:   # prefill chunk: store the degraded KV
                kv = torch.stack([key_states, value_states]).permute(0, 1, 3, 2, 4).unsqueeze(0)
                rec, ratio = sim(kv)
                self.ratios[layer_idx] = ratio
                rec = rec[0].permute(0, 1, 3, 2, 4)
                key_states, value_states = rec[0].contiguous(), rec[1].contiguous()
            return super().update(key_states, value_states, layer_idx, cache_kwargs)

    cache = _SimCache()
    cache.ratios = {}
    return cache
