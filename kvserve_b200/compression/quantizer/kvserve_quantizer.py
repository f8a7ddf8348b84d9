"""Hybrid-precision min-max quantiser (behaviour of
kvserve_v1/compression/quantizer/kvserve_quantizer.py and split_func.py).

A layer's K and V heads are split into a low- and a high-precision group —
by head score (``split_type="head"``) or by layer (``"layer"``) — quantised
with their own ``*_max_value``, and concatenated low group first along the
head axis.  Tensor-parallel ranks slice the head mask to their local heads.
"""
from __future__ import annotations

from typing import Any

import torch

from ..components import Quantizer
from ..heads import get_scores, low_precision_mask, tp_slice_mask
from .minmax import dequantize, quantize


class KVServeQuantizer(Quantizer):
    def __init__(self, **kwargs: Any) -> None:
        self.model_name = kwargs.get("model_name", "Llama-3.1-8B-Instruct")
        self.hybrid_ratio = kwargs.get("hybrid_ratio", 0.3)
        self.high_key_max_value = kwargs.get("high_key_max_value", 16)
        self.high_value_max_value = kwargs.get("high_value_max_value", 16)
        self.low_key_max_value = kwargs.get("low_key_max_value", 12)
        self.low_value_max_value = kwargs.get("low_value_max_value", 12)
        self.axis_key = kwargs.get("axis_key", "channel")
        self.axis_value = kwargs.get("axis_value", "token")
        self.split_type = kwargs.get("split_type", "head")
        self.tensor_parallel_size = kwargs.get("tensor_parallel_size", 1)
        self.tp_rank = kwargs.get("tp_rank", 0)
        self.score_path = kwargs.get("score_path")
        self.num_layers = kwargs.get("num_layers", 0)
        self.num_kv_heads = kwargs.get("num_kv_heads", 0)
        self.validate()
        self.head_scores = get_scores(self.model_name, self.num_layers, self.num_kv_heads, self.score_path)
        self._rebuild_masks()

    def _rebuild_masks(self) -> None:
        self.head_scores_mask = low_precision_mask(self.head_scores, self.hybrid_ratio, "head")
        self.layer_scores_mask = low_precision_mask(self.head_scores, self.hybrid_ratio, "layer")[:, 0].clone()

    def validate(self) -> None:
        if not 0 <= self.hybrid_ratio <= 1:
            raise ValueError(f"hybrid_ratio must be between 0 and 1, got {self.hybrid_ratio}")
        for name in ("low_key_max_value", "low_value_max_value", "high_key_max_value", "high_value_max_value"):
            v = getattr(self, name)
            if not 0 < v < 255:
                raise ValueError(f"{name} must be in (0, 255), got {v}")
        if self.low_key_max_value > self.high_key_max_value:
            raise ValueError("low_key_max_value must not exceed high_key_max_value")
        if self.low_value_max_value > self.high_value_max_value:
            raise ValueError("low_value_max_value must not exceed high_value_max_value")
        for name in ("axis_key", "axis_value"):
            if getattr(self, name) not in ("channel", "token", "tensor"):
                raise ValueError(f"{name} must be 'channel', 'token' or 'tensor'")
        if self.split_type not in ("head", "layer"):
            raise ValueError(f"split_type must be 'head' or 'layer', got {self.split_type}")

    def update_params(self, **kwargs: Any) -> None:
        old_ratio = self.hybrid_ratio
        for key, value in kwargs.items():
            if hasattr(self, key) and key not in ("head_scores", "head_scores_mask", "layer_scores_mask"):
                setattr(self, key, value)
        self.validate()
        if self.hybrid_ratio != old_ratio:
            self._rebuild_masks()

    def head_mask(self, num_heads: int) -> torch.Tensor:
        return tp_slice_mask(self.head_scores_mask, num_heads, self.tp_rank, self.tensor_parallel_size)

    def _split(self, layer_id: int, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        if self.split_type == "head":
            m = self.head_mask(x.shape[2])[layer_id].to(x.device)
            return x[:, :, m, :], x[:, :, ~m, :]
        empty = torch.zeros(0, dtype=x.dtype, device=x.device)
        return (x, empty) if bool(self.layer_scores_mask[layer_id]) else (empty, x)

    def quantize(self, layer_id: int, tensor: torch.Tensor, **kwargs: Any) -> tuple[torch.Tensor, dict]:
        keys, values = tensor[0], tensor[1]
        lk, hk = self._split(layer_id, keys)
        lv, hv = self._split(layer_id, values)
        hk, hkm = quantize(self.high_key_max_value, hk, self.axis_key)
        hv, hvm = quantize(self.high_value_max_value, hv, self.axis_value)
        lk, lkm = quantize(self.low_key_max_value, lk, self.axis_key)
        lv, lvm = quantize(self.low_value_max_value, lv, self.axis_value)
        if self.split_type == "head":
            keys = torch.cat([lk, hk], dim=2)
            values = torch.cat([lv, hv], dim=2)
        else:
            keys = lk if lk.numel() else hk
            values = lv if lv.numel() else hv
        meta = {"high_key_meta": hkm, "high_value_meta": hvm, "low_key_meta": lkm, "low_value_meta": lvm,
                "original_dtype": str(tensor.dtype).replace("torch.", "")}
        return torch.stack([keys, values], dim=0), meta

    def _restore(self, layer_id: int, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        if self.split_type == "head":
            n_low = int(self.head_mask(x.shape[2])[layer_id].sum())
            return x[:, :, :n_low, :], x[:, :, n_low:, :]
        empty = torch.zeros(0, dtype=x.dtype, device=x.device)
        return (x, empty) if bool(self.layer_scores_mask[layer_id]) else (empty, x)

    def _reconstruct(self, layer_id: int, low: torch.Tensor, high: torch.Tensor, heads: int) -> torch.Tensor:
        if self.split_type == "head":
            m = self.head_mask(heads)[layer_id].to(low.device if low.numel() else high.device)
            out = torch.cat([low, high], dim=2)
            out[:, :, m, :] = low
            out[:, :, ~m, :] = high
            return out
        return low if low.numel() else high

    def dequantize(self, layer_id: int, tensor: torch.Tensor, meta: Any, **kwargs: Any) -> torch.Tensor:
        heads = tensor.shape[3]
        lk, hk = self._restore(layer_id, tensor[0])
        lv, hv = self._restore(layer_id, tensor[1])
        hk = dequantize(hk, meta["high_key_meta"])
        hv = dequantize(hv, meta["high_value_meta"])
        lk = dequantize(lk, meta["low_key_meta"])
        lv = dequantize(lv, meta["low_value_meta"])
        keys = self._reconstruct(layer_id, lk, hk, heads)
        values = self._reconstruct(layer_id, lv, hv, heads)
        return torch.stack([keys, values], dim=0)
