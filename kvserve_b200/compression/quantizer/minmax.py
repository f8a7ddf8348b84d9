"""Min-max quantisation with the reference's ``max_value`` semantics
(kvserve_v1/compression/quantizer/quantizer_func.py:9-113), computed in the
tensor's own dtype exactly as the reference does:

    scale = clamp(max - min, 1e-5) / (max_value - 1)
    q     = clamp(round((x - min) / scale), 0, max_value)        (uint8)
    x'    = q * scale + min

Axes of a ``[num_blocks, block_size, num_heads, head_size]`` tensor:
``channel`` reduces dims (0, 1) (per head and channel), ``token`` reduces
(2, 3) (per token, over every head of the section) and ``tensor`` all dims.
Note the inclusive clamp: the alphabet has ``max_value + 1`` symbols.
"""
from __future__ import annotations

from typing import Any

import torch

_AXES = {"channel": [0, 1], "token": [2, 3], "tensor": [0, 1, 2, 3]}


def quantize(max_value: int, tensor: torch.Tensor, axis: str) -> tuple[torch.Tensor, dict[str, Any]]:
    dtype_name = str(tensor.dtype).replace("torch.", "")
    if tensor.numel() == 0:
        return tensor.to(torch.uint8), {"min_val": None, "quant_scale": None,
                                        "original_dtype": dtype_name, "quant_dtype": "uint8"}
    if axis not in _AXES:
        raise ValueError(f"Invalid axis: {axis}")
    dims = _AXES[axis]
    mx = torch.amax(tensor, dim=dims, keepdim=True)
    mn = torch.amin(tensor, dim=dims, keepdim=True)
    scale = (mx - mn).clamp_(min=1e-5).div_(max_value - 1)
    q = tensor.sub(mn).div_(scale).round_().clamp_(0, max_value).to(torch.uint8)
    return q, {"min_val": mn.to(tensor.dtype), "quant_scale": scale.to(tensor.dtype),
               "original_dtype": dtype_name, "quant_dtype": "uint8"}


def dequantize(q: torch.Tensor, meta: dict[str, Any]) -> torch.Tensor:
    dtype = getattr(torch, meta.get("original_dtype", "bfloat16"))
    if meta.get("min_val") is None:
        return q.to(dtype)
    return q.to(dtype) * meta["quant_scale"] + meta["min_val"]
