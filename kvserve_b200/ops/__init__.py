"""Python front-end of the hand-written sm_100a kernels.

Every function here launches a kernel of ``kvserve_b200._C`` on the current
CUDA stream; none of them synchronises the host.  Device-side failures
(a bounded wait that timed out, a malformed frame) are recorded in per-device
status words and surfaced by :func:`check_device_status`.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from ._ext import ext, available, ExtensionMissing

__all__ = [
    "ext", "available", "ExtensionMissing", "linear", "gemm", "gemv", "rmsnorm", "rope_qkv",
    "silu_mul", "gemm_silu", "gemm_qkv_rope", "interleave_gate_up", "GATE_UP_BLOCK", "embedding", "argmax", "flash_prefill", "paged_decode_attention",
    "device_status", "check_device_status", "STATUS_NAMES",
]

STATUS_NAMES = {0: "ok", 1: "timeout", 2: "bad header", 3: "bad symbol", 4: "bad size"}
GEMV_MAX_M = 8

_status: dict[int, torch.Tensor] = {}

_DTYPE_CODES = {torch.uint8: 0, torch.int8: 1, torch.int16: 2, torch.int32: 3, torch.int64: 4,
                torch.float16: 5, torch.float32: 6, torch.float64: 7, torch.bool: 11, torch.bfloat16: 15}


_launches = [0]


def count_launches(n: int = 1) -> None:
    """Book-keeping of kernel launches issued through this package (eager
    calls; CUDA-graph replays are accounted by their owners)."""
    _launches[0] += n


def launches() -> int:
    return _launches[0]


def dtype_code(dtype: torch.dtype) -> int:
    """c10::ScalarType code of ``dtype`` (for tensors wrapped around raw pointers)."""
    return _DTYPE_CODES[dtype]


def _dev_index(device) -> int:
    if device is None:
        return torch.cuda.current_device()
    if isinstance(device, int):
        return device
    d = torch.device(device)
    return d.index if d.index is not None else torch.cuda.current_device()


def device_status(device: torch.device | int | None = None) -> torch.Tensor:
    """The int32 status word that kernels on ``device`` report failures into."""
    idx = _dev_index(device)
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def check_device_status(device=None, reset: bool = True) -> None:
    """Raise if any kernel on ``device`` recorded an error (synchronises)."""
    st = device_status(device)
    code = int(st[0].item())
    if code != 0:
        if reset:
            st.zero_()
        raise RuntimeError(f"kvserve_b200 device status: {STATUS_NAMES.get(code, code)}")


def gemm(a: torch.Tensor, b: torch.Tensor, out: Optional[torch.Tensor] = None,
         residual: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``out = a @ b.T (+ bias) (+ residual)`` on tcgen05 tensor cores (bf16 in/out, fp32 acc)."""
    if out is None:
        out = torch.empty((a.shape[0], b.shape[0]), dtype=a.dtype, device=a.device)
    count_launches(1)
    ext().gemm_bf16(a, b, out, residual, bias, device_status(a.device))
    return out


def gemv(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
         bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``out = x @ w.T (+ bias)`` for at most 8 rows (weight-streaming kernel)."""
    if out is None:
        out = torch.empty((x.shape[0], w.shape[0]), dtype=x.dtype, device=x.device)
    count_launches(1)
    ext().gemv_bf16(x, w, out, bias)
    return out


def linear(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
           bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """nn.Linear: the weight-streaming GEMV for decode-size batches, the
    tcgen05 tile GEMM otherwise."""
    x2 = x.reshape(-1, x.shape[-1])
    if x2.shape[0] <= GEMV_MAX_M:
        y = gemv(x2, w, out, bias)
    else:
        y = gemm(x2, w, out, bias=bias)
    return y.view(*x.shape[:-1], w.shape[0])


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float,
            residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """RMSNorm; with ``residual`` the input is first added into it (in place)."""
    if out is None:
        out = torch.empty_like(x)
    count_launches(1)
    ext().rmsnorm(x, residual, weight, out, eps)
    return out


def rope_qkv(qkv: torch.Tensor, num_q_heads: int, num_kv_heads: int, head_dim: int,
             positions: torch.Tensor, cos_sin: torch.Tensor, k_dst: Optional[torch.Tensor] = None,
             v_dst: Optional[torch.Tensor] = None, slot_mapping: Optional[torch.Tensor] = None,
             slot_base: int = 0) -> None:
    """Rotary embedding on q/k of a fused QKV tensor (in place) and copy of the
    rotated k and of v into ``k_dst``/``v_dst`` (``[slots, Hkv, D]`` views)."""
    if k_dst is not None:
        tok_stride, head_stride = k_dst.stride(0), k_dst.stride(1)
    else:
        tok_stride, head_stride = 0, 0
    count_launches(1)
    ext().rope_qkv(qkv, num_q_heads, num_kv_heads, head_dim, positions, cos_sin, k_dst, v_dst,
                   tok_stride, head_stride, slot_mapping, slot_base)


def silu_mul(gate_up: torch.Tensor, out: Optional[torch.Tensor] = None, block: int = 0) -> torch.Tensor:
    """``silu(gate) * up``.  ``block == 0``: ``gate_up = [gate | up]``;
    ``block > 0``: gate and up columns interleaved in blocks of ``block``
    (the layout of :func:`interleave_gate_up`)."""
    inter = gate_up.shape[-1] // 2
    if out is None:
        out = torch.empty((*gate_up.shape[:-1], inter), dtype=gate_up.dtype, device=gate_up.device)
    count_launches(1)
    ext().silu_mul(gate_up, out, int(block))
    return out


GATE_UP_BLOCK = 128


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor, block: int = GATE_UP_BLOCK) -> torch.Tensor:
    """Stack ``gate``/``up`` weights ``[I, K]`` as ``[2I, K]`` with rows
    interleaved in blocks of ``block`` (gate block b, then up block b), the
    operand layout of :func:`gemm_silu`."""
    I, K = gate.shape
    if I % block:
        raise ValueError("intermediate size must be a multiple of the interleave block")
    return torch.stack([gate.view(I // block, block, K), up.view(I // block, block, K)], 1).reshape(2 * I, K)


def gemm_qkv_rope(a: torch.Tensor, w_qkv: torch.Tensor, num_q_heads: int, num_kv_heads: int,
                  positions: torch.Tensor, cos_sin: torch.Tensor, bias: Optional[torch.Tensor] = None,
                  k_dst: Optional[torch.Tensor] = None, v_dst: Optional[torch.Tensor] = None,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused QKV projection (head_dim 128): ``a @ w_qkv^T (+ bias)`` with the
    rotary embedding applied to the q and k heads in the GEMM epilogue and
    the rotated k / the v rows also written to ``k_dst``/``v_dst``
    (``[tokens, kv_heads, 128]`` views) — the same result as :func:`linear`
    followed by :func:`rope_qkv`."""
    if out is None:
        out = torch.empty((a.shape[0], w_qkv.shape[0]), dtype=a.dtype, device=a.device)
    count_launches(1)
    ext().gemm_qkv_rope_bf16(a, w_qkv, out, bias, cos_sin, positions, int(num_q_heads), int(num_kv_heads), k_dst,
                             v_dst, device_status(a.device))
    return out


def gemm_silu(a: torch.Tensor, w_gate_up: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``silu(a @ gate^T) * (a @ up^T)`` in one tcgen05 GEMM whose epilogue
    applies the activation; ``w_gate_up`` is ``[2I, K]`` in the
    :func:`interleave_gate_up` layout."""
    if out is None:
        out = torch.empty((a.shape[0], w_gate_up.shape[0] // 2), dtype=a.dtype, device=a.device)
    count_launches(1)
    ext().gemm_silu_bf16(a, w_gate_up, out, device_status(a.device))
    return out


def embedding(ids: torch.Tensor, table: torch.Tensor, vocab_begin: int = 0,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty((ids.numel(), table.shape[1]), dtype=table.dtype, device=table.device)
    count_launches(1)
    ext().embedding(ids, table, out, vocab_begin)
    return out


def argmax(logits: torch.Tensor, index_offset: int = 0, out_val: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    count_launches(1)
    ext().argmax_rows(logits, out, out_val, index_offset)
    return out


def flash_prefill(qkv: torch.Tensor, num_q_heads: int, num_kv_heads: int,
                  scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                  kstages: int = 0, poly: int = 0) -> torch.Tensor:
    """Causal GQA attention over a fused (already rotated) QKV tensor, head_dim 128.
    ``kstages`` (2 or 3) sets the depth of the kernel's K-tile ring (0:
    ``KVSERVE_FLASH_KSTAGES``, default 2); ``poly`` picks which of every 8
    exponential pairs run as a polynomial on the FMA pipes instead of the
    MUFU (bit mask 0x11, 0x55 or 0xFF; 0x100 = none, the default)."""
    d = 128
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty((qkv.shape[0], num_q_heads * d), dtype=qkv.dtype, device=qkv.device)
    count_launches(1)
    ext().flash_prefill(qkv, num_q_heads, num_kv_heads, scale, out, device_status(qkv.device), int(kstages), int(poly))
    return out


def paged_decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_tables: torch.Tensor, ctx_lens: torch.Tensor, max_ctx: int,
                           scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                           scratch: Optional[tuple[torch.Tensor, torch.Tensor]] = None) -> torch.Tensor:
    """Single-token GQA attention over paged K/V (``[num_blocks, block_size, Hkv, D]``)."""
    b, hq, d = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty_like(q)
    splits = ext().paged_decode_splits(b, k_cache.shape[2], max_ctx)
    if scratch is None:
        part_o = torch.empty(b * hq * splits * d, dtype=torch.float32, device=q.device)
        part_ml = torch.empty(b * hq * splits * 2, dtype=torch.float32, device=q.device)
    else:
        part_o, part_ml = scratch
    count_launches(2 if splits > 1 else 1)
    ext().paged_decode_attention(q, k_cache, v_cache, block_tables, ctx_lens, max_ctx, scale, out,
                                 part_o, part_ml, splits)
    return out
