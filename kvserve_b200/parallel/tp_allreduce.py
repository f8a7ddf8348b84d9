"""Fused GEMM + tensor-parallel all-reduce over NVLink peer memory.

A row-parallel projection (attention output, MLP down) is followed in plain
TP by an all-reduce of its [M, N] result.  Here both are ONE launch of the
tcgen05 GEMM (epilogue mode 3 of ``csrc/gemm_sm100.cu``): each output tile
is reduced by one owner rank, the other ranks store their bf16 partial tile
into the owner's staging memory over NVLink while their tensor cores go on
with the next tiles, and the owner writes the reduced tile into every rank's
output.  NCCL stays for the small decode-size reductions inside CUDA graphs.

Every rank of the TP group holds one device region, exported through CUDA
IPC and mapped by its peers:

    out    [max_tokens, hidden] bf16            the all-reduced result
    stage  [world-1][max_tiles][128*256] bf16   partial tiles, one slot per source
    flags  [world-1][max_tiles] + [max_tiles]   u32 partial / final epochs

Role in the reference: the TP model math and its all-reduce are vLLM's there
(row-parallel linear layers, vllm/model_executor/layers/linear.py); the
reference adds only the KV side (kvserve_v1/connector/compressed_kv_connector.py:192-204
opens one channel per TP rank).
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops

TILE_M, TILE_N = 128, 256
MAX_RANKS = 8


def fused_allreduce_enabled() -> bool:
    return os.environ.get("KVSERVE_FUSED_ALLREDUCE", "1").strip().lower() not in {"0", "false", "no", "off"}


def workspace_layout(world: int, max_tokens: int, hidden: int) -> dict:
    """Byte offsets of the three parts of one rank's region (16-byte aligned)."""
    if not 1 <= world <= MAX_RANKS:
        raise ValueError(f"fused all-reduce supports 1..{MAX_RANKS} ranks")
    if hidden % TILE_N:
        raise ValueError(f"hidden size must be a multiple of {TILE_N}")
    max_tiles = -(-max_tokens // TILE_M) * (hidden // TILE_N)
    align = lambda n: (n + 255) // 256 * 256  # noqa: E731
    out_bytes = align(max_tokens * hidden * 2)
    stage_bytes = align((world - 1) * max_tiles * TILE_M * TILE_N * 2)
    flag_bytes = align(world * max_tiles * 4)
    return dict(max_tiles=max_tiles, out=0, stage=out_bytes, flags=out_bytes + stage_bytes,
                flag_bytes=flag_bytes, total=out_bytes + stage_bytes + flag_bytes)


class TPAllReduce:
    """One rank's handle on the symmetric workspace of its TP group."""

    def __init__(self, world: int, rank: int, max_tokens: int, hidden: int, device: torch.device,
                 timeout_s: Optional[float] = None):
        self.world, self.rank = world, rank
        self.max_tokens, self.hidden = max_tokens, hidden
        self.device = torch.device(device)
        self.lay = workspace_layout(world, max_tokens, hidden)
        self.max_tiles = self.lay["max_tiles"]
        if timeout_s is None:
            timeout_s = float(os.environ.get("KVSERVE_TP_TIMEOUT_S", "10"))
        self.timeout_ns = int(timeout_s * 1e9)
        self.epoch = 0
        with torch.cuda.device(self.device):
            self.base = ops.ext().dev_alloc(self.lay["total"])
            flags = ops.ext().tensor_from_ptr(self.base + self.lay["flags"], [self.lay["flag_bytes"] // 4],
                                              ops.dtype_code(torch.int32), self.device.index)
            flags.zero_()
        self._bases = [0] * world
        self._bases[rank] = self.base
        self._opened: list[int] = []
        self.out_ptrs = self.stage_ptrs = self.flag_ptrs = None

    # ------------------------------------------------------------ wiring
    def handle(self) -> bytes:
        return ops.ext().ipc_get_handle(self.base)

    def connect(self, handles: list[Optional[bytes]]) -> None:
        """Map every peer's region (``handles[r]`` for TP rank r; own ignored)."""
        if len(handles) != self.world:
            raise ValueError("one handle per TP rank")
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r != self.rank:
                    self._bases[r] = ops.ext().ipc_open_handle(h)
                    self._opened.append(self._bases[r])
        self.out_ptrs = [b + self.lay["out"] for b in self._bases]
        self.stage_ptrs = [b + self.lay["stage"] for b in self._bases]
        self.flag_ptrs = [b + self.lay["flags"] for b in self._bases]

    def output(self, m: int, n: int) -> torch.Tensor:
        """The [m, n] result view on this rank (shared with the peers)."""
        return ops.ext().tensor_from_ptr(self.base + self.lay["out"], [m, n], ops.dtype_code(torch.bfloat16),
                                         self.device.index)

    # -------------------------------------------------------------- call
    def accepts(self, m: int, n: int) -> bool:
        return (self.out_ptrs is not None and ops.GEMV_MAX_M < m <= self.max_tokens and n <= self.hidden
                and n % TILE_N == 0 and m * n <= self.max_tokens * self.hidden
                and not torch.cuda.is_current_stream_capturing())

    def gemm_allreduce(self, a: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """sum over the TP group of ``a_r @ w_r.T`` (bf16, fp32 accumulate),
        returned on every rank.  Every rank must call it in the same order."""
        a2 = a.reshape(-1, a.shape[-1])
        m, n = a2.shape[0], w.shape[0]
        if m > self.max_tokens or n > self.hidden or n % TILE_N or self.out_ptrs is None:
            raise ValueError(f"gemm_allreduce: [{m}, {n}] does not fit the workspace "
                             f"[{self.max_tokens}, {self.hidden}] (or it is not connected)")
        out = self.output(m, n)
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF or 1
        ops.count_launches(1)
        ops.ext().gemm_allreduce_bf16(a2, w, out, self.out_ptrs, self.stage_ptrs, self.flag_ptrs, self.rank,
                                      self.max_tiles, self.epoch, self.timeout_ns, ops.device_status(a.device))
        return out.view(*a.shape[:-1], n)

    def close(self) -> None:
        with torch.cuda.device(self.device):
            for p in self._opened:
                ops.ext().ipc_close(p)
            self._opened = []
            if self.base:
                ops.ext().dev_free(self.base)
                self.base = 0
        self.out_ptrs = None


def create_tp_allreduce(ctx, max_tokens: int, hidden: int, device: torch.device, participate: bool = True,
                        timeout_s: Optional[float] = None) -> Optional[TPAllReduce]:
    """Collective over ``ctx.cpu_group`` (every rank of the job calls it, in
    the same order): ranks with ``participate`` and ``ctx.tp_size > 1``
    allocate a workspace and map those of the other ranks of their TP group.
    Returns None where no workspace is made (TP 1, not participating, or
    fused reductions switched off)."""
    use = participate and ctx.tp_size > 1 and fused_allreduce_enabled() and hidden % TILE_N == 0 \
        and ctx.tp_size <= MAX_RANKS
    ws = TPAllReduce(ctx.tp_size, ctx.tp_rank, max_tokens, hidden, device, timeout_s) if use else None
    if not ctx.distributed:
        return ws
    mine = (ctx.role, ctx.tp_rank, ws.handle() if ws is not None else None)
    allh: list = [None] * ctx.world_size
    dist.all_gather_object(allh, mine, group=ctx.cpu_group)
    if ws is not None:
        group = {tp: h for role, tp, h in allh if role == ctx.role}
        if len(group) != ctx.tp_size or any(h is None for h in group.values()):
            ws.close()
            ws = None
        else:
            ws.connect([group[r] for r in range(ctx.tp_size)])
    torch.cuda.synchronize(device)   # flags are zero before any peer may write them
    dist.barrier(group=ctx.cpu_group)
    return ws
