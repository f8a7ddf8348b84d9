"""Calibration-free centred Gaussian codebook quantiser (behaviour of
kvserve_v1/compression/quantizer/centered_codebook.py).

Codebook: Lloyd-Max centroids of a standard normal for 1..4 bits, computed
here by Lloyd's fixed-point iteration (centroid = conditional mean of the
Gaussian on each cell; cells bounded by midpoints).
Keys: per (head, channel) over token groups of ``group_size`` tokens;
values: per (head, token) over the head dimension.  Each group gets a mean
(``mean_dtype``) and an RMS scale times ``scale_alpha`` (bf16), optionally
refined by ``scale_refinements`` least-squares steps; symbols are the cell
index of ``(x - mean) / scale``.  CUDA tensors run the sm_100a kernels of
``csrc/codebook.cu`` (one thread per key channel over a token group, one warp
per value row; the reference runs Triton kernels,
kvserve_v1/compression/quantizer/centered_codebook.py:67-161); CPU tensors
run the same arithmetic as vectorised torch ops.
"""
from __future__ import annotations

import math
from functools import lru_cache
from typing import Any

import torch

from ..components import Quantizer


@lru_cache(maxsize=8)
def lloyd_max_gaussian(bits: int, iterations: int = 300) -> tuple[float, ...]:
    levels = 1 << bits
    c = [(i - (levels - 1) / 2) * 4.0 / levels for i in range(levels)]
    phi = lambda x: math.exp(-0.5 * x * x) / math.sqrt(2 * math.pi)  # noqa: E731
    Phi = lambda x: 0.5 * (1.0 + math.erf(x / math.sqrt(2.0)))  # noqa: E731
    for _ in range(iterations):
        edges = [-12.0] + [(a + b) / 2 for a, b in zip(c, c[1:])] + [12.0]
        c = [(phi(edges[i]) - phi(edges[i + 1])) / max(Phi(edges[i + 1]) - Phi(edges[i]), 1e-15)
             for i in range(levels)]
    return tuple(c)


class CenteredCodebookQuantizer(Quantizer):
    _defaults = dict(key_bits=3, value_bits=3, group_size=128, scale_refinements=1, scale_alpha=1.0,
                     mean_dtype="float32")
    supports_out_buffer = True

    def __init__(self, **kwargs: Any) -> None:
        self._config = dict(self._defaults)
        self.update_params(**kwargs)

    def _settings(self, kwargs: dict) -> dict:
        cfg = self._config | {k: v for k, v in kwargs.items() if k in self._defaults}
        for k in ("key_bits", "value_bits"):
            if type(cfg[k]) is not int or not 1 <= cfg[k] <= 4:
                raise ValueError("key_bits/value_bits must be integers in [1, 4]")
        if cfg["group_size"] not in (16, 32, 64, 128, 256):
            raise ValueError("group_size must be 16, 32, 64, 128 or 256")
        if cfg["scale_refinements"] not in (0, 1, 2):
            raise ValueError("scale_refinements must be 0, 1 or 2")
        a = cfg["scale_alpha"]
        if not isinstance(a, (int, float)) or not math.isfinite(a) or a <= 0:
            raise ValueError("scale_alpha must be finite and positive")
        if cfg["mean_dtype"] not in ("bfloat16", "float32"):
            raise ValueError("mean_dtype must be bfloat16 or float32")
        return cfg

    def update_params(self, **kwargs: Any) -> None:
        self._config = self._settings(kwargs)

    @staticmethod
    def _tables(bits: int, device) -> tuple[torch.Tensor, torch.Tensor]:
        c = torch.tensor(lloyd_max_gaussian(bits), dtype=torch.float32, device=device)
        return c, (c[:-1] + c[1:]) / 2

    @staticmethod
    def _check(t: torch.Tensor) -> None:
        if t.ndim != 5 or t.shape[0] != 2:
            raise ValueError("expected KV [2, blocks, tokens, heads, dim]")
        if not 1 <= t.shape[-1] <= 512:
            raise ValueError("supported head dimensions are 1-512")

    def _fit(self, x: torch.Tensor, dim: int, cfg: dict, bits: int):
        """x grouped so that reduction is over ``dim``; returns mean, scale, q."""
        mdt = getattr(torch, cfg["mean_dtype"])
        n = x.shape[dim]
        mean = (x.sum(dim, keepdim=True) / n).to(mdt).float()
        res = x - mean
        scale = (torch.sqrt((res * res).sum(dim, keepdim=True) / n) * cfg["scale_alpha"]).to(torch.bfloat16).float()
        centers, bounds = self._tables(bits, x.device)
        for _ in range(cfg["scale_refinements"]):
            q = torch.bucketize(res / scale.clamp_min(1e-20), bounds)
            c = centers[q]
            scale = ((res * c).sum(dim, keepdim=True) / (c * c).sum(dim, keepdim=True).clamp_min(1e-20))
            scale = scale.clamp_min(0.0).to(torch.bfloat16).float()
        q = torch.bucketize(res / scale.clamp_min(1e-20), bounds)
        return mean, scale, q.to(torch.uint8)

    @staticmethod
    def _cuda_ok(t: torch.Tensor) -> bool:
        return t.is_cuda and t.dtype in (torch.bfloat16, torch.float16, torch.float32)

    def _quantize_cuda(self, tensor: torch.Tensor, cfg: dict, out: torch.Tensor) -> list[dict]:
        from ... import ops
        _, blocks, tokens, heads, dim = tensor.shape
        total, group = blocks * tokens, cfg["group_size"]
        mdt = getattr(torch, cfg["mean_dtype"])
        ng = (total + group - 1) // group
        parts = []
        for part, bits in ((0, cfg["key_bits"]), (1, cfg["value_bits"])):
            x = tensor[part].reshape(total, heads, dim).contiguous()
            shape = (heads, ng, dim) if part == 0 else (heads, total)
            mean = torch.empty(shape, dtype=mdt, device=tensor.device)
            scale = torch.empty(shape, dtype=torch.bfloat16, device=tensor.device)
            q = out[part].view(total, heads, dim) if out[part].is_contiguous() else \
                torch.empty((total, heads, dim), dtype=torch.uint8, device=tensor.device)
            centers = torch.tensor(lloyd_max_gaussian(bits), dtype=torch.float32)
            ops.count_launches(1)
            ops.ext().codebook_quantize(x, part, group, cfg["scale_refinements"], float(cfg["scale_alpha"]),
                                        centers, q, mean, scale)
            if q.data_ptr() != out[part].data_ptr():
                out[part].copy_(q.view(blocks, tokens, heads, dim))
            parts.append(dict(mean=mean, scale=scale))
        return parts

    def quantize(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any) -> tuple[torch.Tensor, dict]:
        self._check(tensor)
        cfg = self._settings({k: v for k, v in kwargs.items() if k != "out"})
        _, blocks, tokens, heads, dim = tensor.shape
        total, group = blocks * tokens, cfg["group_size"]
        out = kwargs.get("out")
        if out is None:
            out = torch.empty(tensor.shape, dtype=torch.uint8, device=tensor.device)
        meta = dict(format="centered_codebook_v1", config=cfg,
                    original_dtype=str(tensor.dtype).replace("torch.", ""))
        if self._cuda_ok(tensor):
            return out, dict(meta, parts=self._quantize_cuda(tensor, cfg, out))
        parts = []
        mdt = getattr(torch, cfg["mean_dtype"])
        # keys: [total, heads, dim] -> groups of tokens
        k = tensor[0].reshape(total, heads, dim).float()
        ng = (total + group - 1) // group
        pad = ng * group - total
        kp = torch.nn.functional.pad(k, (0, 0, 0, 0, 0, pad)) if pad else k
        kg = kp.view(ng, group, heads, dim)
        # per-group token counts (the last group may be partial)
        counts = torch.full((ng, 1, 1, 1), float(group), device=k.device)
        counts[-1] = float(group - pad)
        valid = torch.ones(ng * group, device=k.device)
        if pad:
            valid[total:] = 0
        valid = valid.view(ng, group, 1, 1)
        mean = ((kg * valid).sum(1, keepdim=True) / counts).to(mdt).float()
        res = (kg - mean) * valid
        scale = (torch.sqrt((res * res).sum(1, keepdim=True) / counts) * cfg["scale_alpha"]).to(torch.bfloat16).float()
        centers, bounds = self._tables(cfg["key_bits"], k.device)
        for _ in range(cfg["scale_refinements"]):
            c = centers[torch.bucketize(res / scale.clamp_min(1e-20), bounds)] * valid
            scale = ((res * c).sum(1, keepdim=True) / (c * c).sum(1, keepdim=True).clamp_min(1e-20))
            scale = scale.clamp_min(0.0).to(torch.bfloat16).float()
        qk = torch.bucketize(res / scale.clamp_min(1e-20), bounds).to(torch.uint8)
        out[0].copy_(qk.view(ng * group, heads, dim)[:total].view(blocks, tokens, heads, dim))
        parts.append(dict(mean=mean.view(ng, heads, dim).permute(1, 0, 2).contiguous().to(mdt),
                          scale=scale.view(ng, heads, dim).permute(1, 0, 2).contiguous().to(torch.bfloat16)))
        # values: per (token, head) over dim
        v = tensor[1].reshape(total, heads, dim).float()
        mean_v, scale_v, qv = self._fit(v, 2, cfg, cfg["value_bits"])
        out[1].copy_(qv.view(blocks, tokens, heads, dim))
        parts.append(dict(mean=mean_v.view(total, heads).t().contiguous().to(mdt),
                          scale=scale_v.view(total, heads).t().contiguous().to(torch.bfloat16)))
        return out, dict(format="centered_codebook_v1", config=cfg,
                         original_dtype=str(tensor.dtype).replace("torch.", ""), parts=parts)

    def dequantize(self, layer_id: int, tensor: torch.Tensor, meta: Any, **kwargs: Any) -> torch.Tensor:
        self._check(tensor)
        if tensor.dtype != torch.uint8 or meta.get("format") != "centered_codebook_v1":
            raise ValueError("invalid centered-codebook payload or format")
        if set(meta.get("config", {})) != set(self._defaults) or len(meta.get("parts", [])) != 2:
            raise ValueError("incomplete centered-codebook metadata")
        cfg = self._settings(meta["config"])
        dtype = getattr(torch, meta["original_dtype"])
        _, blocks, tokens, heads, dim = tensor.shape
        total, group = blocks * tokens, cfg["group_size"]
        out = torch.empty(tensor.shape, dtype=dtype, device=tensor.device)
        if tensor.is_cuda and dtype in (torch.bfloat16, torch.float16, torch.float32):
            from ... import ops
            status = torch.zeros(4, dtype=torch.int32, device=tensor.device)
            for part, bits in ((0, cfg["key_bits"]), (1, cfg["value_bits"])):
                p = meta["parts"][part]
                centers = torch.tensor(lloyd_max_gaussian(bits), dtype=torch.float32)
                ops.count_launches(1)
                ops.ext().codebook_dequantize(tensor[part].reshape(total, heads, dim).contiguous(), part, group,
                                              centers, p["mean"].contiguous(), p["scale"].contiguous(),
                                              out[part].view(total, heads, dim), status)
            if int(status[0].item()) != 0:
                raise ValueError("invalid centered-codebook symbol")
            return out
        # keys
        centers, _ = self._tables(cfg["key_bits"], tensor.device)
        q = tensor[0].reshape(total, heads, dim).long()
        if int(q.max()) >= (1 << cfg["key_bits"]) if q.numel() else False:
            raise ValueError("invalid centered-codebook symbol")
        gidx = torch.arange(total, device=tensor.device) // group
        mean = meta["parts"][0]["mean"].float().permute(1, 0, 2)[gidx]   # [total, heads, dim]
        scale = meta["parts"][0]["scale"].float().permute(1, 0, 2)[gidx]
        out[0].copy_((centers[q] * scale + mean).view(blocks, tokens, heads, dim))
        centers, _ = self._tables(cfg["value_bits"], tensor.device)
        q = tensor[1].reshape(total, heads, dim).long()
        if int(q.max()) >= (1 << cfg["value_bits"]) if q.numel() else False:
            raise ValueError("invalid centered-codebook symbol")
        mean = meta["parts"][1]["mean"].float().t()[:, :, None]
        scale = meta["parts"][1]["scale"].float().t()[:, :, None]
        out[1].copy_((centers[q] * scale + mean).view(blocks, tokens, heads, dim))
        return out
