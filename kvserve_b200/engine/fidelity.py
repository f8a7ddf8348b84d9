"""Reconstruction error of a transfer profile on synthetic KV.

The synthetic KV has the distribution of the benchmark's first configuration:
values N(0, 1); keys N(0, 1) with 4 fixed channels per head scaled by 8
(outlier channels, the case per-channel key quantisation is for).  The same
generator feeds this framework's frame kernels here and the reference's
modular pipeline in the reference arm, so the two reconstruction errors are
measured on identical data.

``frame_round_trip`` runs the product path: the fused encode kernel writes
each layer's frame into device memory, the fused decode kernel writes it back
into a paged cache, and the error is taken against the bf16 input.
"""
from __future__ import annotations

from typing import Optional

import torch


def synthetic_kv(layers: int, tokens: int, heads: int, dim: int, seed: int = 0,
                 device: Optional[torch.device] = None) -> torch.Tensor:
    """``[layers, 2, tokens, heads, dim]`` bf16 (index 0 keys, 1 values)."""
    g = torch.Generator().manual_seed(seed)
    kv = torch.randn((layers, 2, tokens, heads, dim), generator=g)
    outliers = torch.randperm(dim, generator=g)[:4]
    kv[:, 0, :, :, outliers] *= 8.0
    kv = kv.to(torch.bfloat16)
    return kv.to(device) if device is not None else kv


def error_stats(ref: torch.Tensor, out: torch.Tensor) -> dict:
    """MSE and relative MSE (error power / signal power) overall and for K, V;
    ``ref``/``out`` are ``[L, 2, ...]``."""
    r = ref.float()
    e = (out.float() - r).pow(2)
    stats = {"mse": e.mean().item(), "rel_mse": (e.sum() / r.pow(2).sum()).item()}
    for i, name in enumerate(("k", "v")):
        stats[f"{name}_mse"] = e[:, i].mean().item()
        stats[f"{name}_rel_mse"] = (e[:, i].sum() / r[:, i].pow(2).sum()).item()
    return {k: float(f"{v:.6g}") for k, v in stats.items()}


def frame_round_trip(xfer, kv: torch.Tensor, block_size: int = 16) -> torch.Tensor:
    """Encode every layer of ``kv`` ``[L, 2, T, H, D]`` (CUDA, bf16) with the
    fused frame kernels of ``xfer`` (a :class:`~kvserve_b200.engine.transfer.KVTransfer`
    with at least ``L`` layers), decode into a paged cache, return the
    reconstruction in the input's layout."""
    from .. import ops
    L, _, T, H, D = kv.shape
    dev = kv.device
    nblk = (T + block_size - 1) // block_size
    cache = torch.zeros((xfer.L, 2, nblk, block_size, H, D), dtype=torch.bfloat16, device=dev)
    table = torch.arange(nblk, dtype=torch.int32, device=dev)
    status = ops.device_status(dev)
    frame = torch.empty(max(xfer.frame_stride, 256), dtype=torch.uint8, device=dev)
    for l in range(L):
        k, v = kv[l, 0].contiguous(), kv[l, 1].contiguous()
        xfer.encode(l, k, v, frame.data_ptr(), 0, 1)
        xfer.ingest_layer(l, T, frame.data_ptr(), cache, table, status, 1)
    torch.cuda.synchronize(dev)
    if int(status[0].item()) != 0:
        raise RuntimeError(f"frame round trip failed: status {int(status[0].item())}")
    return cache[:L].reshape(L, 2, nblk * block_size, H, D)[:, :, :T]


def measure_profile(profile, layers: int, tokens: int, heads: int, dim: int, device: torch.device,
                    seed: int = 0) -> dict:
    """Reconstruction error and compression ratio of ``profile`` (a
    :class:`~kvserve_b200.engine.transfer.TransferProfile`) on ``layers``
    synthetic layers."""
    from .transfer import KVTransfer
    xfer = KVTransfer(profile, layers, heads, heads, dim, 0, 1, device, tokens, profile.score_model)
    kv = synthetic_kv(layers, tokens, heads, dim, seed, device)
    out = frame_round_trip(xfer, kv)
    st = error_stats(kv, out)
    st.update({"compression_ratio": round(xfer.raw_bytes(tokens) / xfer.payload_bytes(tokens), 3),
               "layers": layers, "tokens": tokens, "kv_heads": heads, "head_dim": dim,
               "data": "synthetic: V ~ N(0,1), K ~ N(0,1) with 4 outlier channels x8 per head, seed %d" % seed})
    return st
