"""Decode-step collectives fused into the projection kernels (NVLink peer memory).

A tensor-parallel decode step (M <= 8 tokens) has two all-reduces per layer
(attention output and MLP down) and a greedy argmax over the vocabulary-
parallel LM head.  With NCCL each is a separate launch whose latency, not
its bytes, sets the cost.  Here they are epilogues of the projections that
produce them (``csrc/decode_fused.cu``):

* ``gemv_allreduce``: each CTA stores its fp32 partial rows into every TP
  rank's staging memory as 64-bit "LL" words (flag in the high half, value
  in the low half; an aligned 64-bit store is single-copy atomic, so no fence
  or separate flag is needed), polls its own staging for the peers' words
  and sums in rank order (every rank gets bitwise the same result);
* ``gemv_argmax``: LM head + greedy argmax, with an exchange of each rank's
  best (value, index) as two LL words — the logits never leave the kernel;
* ``bump``: the step epoch that tags the words, advanced once per step.

Every rank of a TP group holds one device region, exported through CUDA IPC
and mapped by its peers:

    stage  [2 parities][world][8 tokens][hidden]   u64   LL partial rows
    aslot  [2][world][8 tokens][2]                 u64   LL argmax candidates

The reference serves decode with vLLM, whose row-parallel layers call an
NCCL all-reduce; this module is the standalone engine's replacement.
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops

MAX_RANKS = 8
MAX_TOKENS = 8
ROWS_PER_CTA = 16


def decode_fusion_enabled() -> bool:
    return os.environ.get("KVSERVE_DECODE_FUSED_AR", "1").strip().lower() not in {"0", "false", "no", "off"}


def region_layout(world: int, hidden: int) -> dict:
    """Byte offsets of one rank's region (256-byte aligned parts)."""
    if not 1 <= world <= MAX_RANKS:
        raise ValueError(f"decode collectives support 1..{MAX_RANKS} ranks")
    if hidden % ROWS_PER_CTA:
        raise ValueError(f"hidden size must be a multiple of {ROWS_PER_CTA}")
    align = lambda n: (n + 255) // 256 * 256  # noqa: E731
    stage = align(2 * world * MAX_TOKENS * hidden * 8)
    aslot = align(2 * world * MAX_TOKENS * 2 * 8)
    return dict(stage=0, aslot=stage, total=stage + aslot, stage_ld=hidden)


class DecodeCollectives:
    """One rank's handle on the decode-step collective workspace of its TP
    group (world 1 keeps only the fused LM-head argmax)."""

    def __init__(self, world: int, rank: int, hidden: int, vocab_local: int, num_sites: int, device,
                 timeout_s: Optional[float] = None):
        self.world, self.rank, self.hidden = world, rank, hidden
        self.device = torch.device(device)
        self.num_sites = num_sites
        self.lay = region_layout(world, hidden)
        if timeout_s is None:
            timeout_s = float(os.environ.get("KVSERVE_TP_TIMEOUT_S", "10"))
        self.timeout_ns = int(timeout_s * 1e9)
        dev = self.device
        self.epoch = torch.zeros(1, dtype=torch.int32, device=dev)
        self.status = ops.device_status(dev)
        grid = -(-vocab_local // ROWS_PER_CTA)
        self.part_val = torch.empty(MAX_TOKENS * grid, dtype=torch.float32, device=dev)
        self.part_idx = torch.empty(MAX_TOKENS * grid, dtype=torch.int32, device=dev)
        self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
        self.base = 0
        self._opened: list[int] = []
        self._bases: list[int] = []
        if world > 1:
            with torch.cuda.device(dev):
                self.base = ops.ext().dev_alloc(self.lay["total"])
                ops.ext().tensor_from_ptr(self.base, [self.lay["total"] // 4], ops.dtype_code(torch.int32),
                                          dev.index).zero_()
            self._bases = [0] * world
            self._bases[rank] = self.base
        self.connected = world == 1

    # ------------------------------------------------------------ wiring
    def handle(self) -> Optional[bytes]:
        return ops.ext().ipc_get_handle(self.base) if self.base else None

    def connect(self, handles: list) -> None:
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r != self.rank:
                    self._bases[r] = ops.ext().ipc_open_handle(h)
                    self._opened.append(self._bases[r])
        self.connected = True

    def _ptrs(self, part: str) -> list[int]:
        return [b + self.lay[part] for b in self._bases]

    # -------------------------------------------------------------- calls
    def gemv_allreduce(self, x: torch.Tensor, w: torch.Tensor, site: int) -> torch.Tensor:
        """``sum over ranks of x_r @ w_r.T`` for a decode batch (M <= 8), on
        every rank, in one launch.  Every rank calls it with the same site."""
        x2 = x.reshape(-1, x.shape[-1])
        y = torch.empty((x2.shape[0], w.shape[0]), dtype=torch.bfloat16, device=x.device)
        ops.count_launches(1)
        ops.ext().gemv_allreduce_bf16(x2, w, y, self._ptrs("stage"), self.rank, site, self.num_sites, self.epoch,
                                      self.lay["stage_ld"], self.timeout_ns, self.status)
        return y

    def greedy(self, h: torch.Tensor, lm_head: torch.Tensor, vocab_begin: int, site: int) -> torch.Tensor:
        """Greedy next token (int32 [M]) over the vocab-parallel LM head."""
        out = torch.empty(h.shape[0], dtype=torch.int32, device=h.device)
        slots = self._ptrs("aslot") if self.world > 1 else []
        ops.count_launches(1)
        ops.ext().gemv_argmax_bf16(h, lm_head, out, self.part_val, self.part_idx, self.counter, vocab_begin,
                                   slots, self.rank, site, self.num_sites, self.epoch, self.timeout_ns,
                                   self.status)
        return out

    def bump(self) -> None:
        if self.world > 1:
            ops.count_launches(1)
            ops.ext().decode_epoch_bump(self.epoch)

    def close(self) -> None:
        with torch.cuda.device(self.device):
            for p in self._opened:
                ops.ext().ipc_close(p)
            self._opened = []
            if self.base:
                ops.ext().dev_free(self.base)
                self.base = 0
        self.connected = False


def create_decode_collectives(ctx, hidden: int, vocab_local: int, num_sites: int, device,
                              participate: bool = True,
                              timeout_s: Optional[float] = None) -> Optional[DecodeCollectives]:
    """Collective over ``ctx.cpu_group`` (every rank of the job calls it, in
    the same order): ranks with ``participate`` build a workspace and map
    those of the other ranks of their TP group.  Returns None where the fused
    path is off or the geometry does not fit (the model then keeps NCCL)."""
    use = (participate and decode_fusion_enabled() and hidden % ROWS_PER_CTA == 0
           and ctx.tp_size <= MAX_RANKS)
    ws = DecodeCollectives(ctx.tp_size, ctx.tp_rank, hidden, vocab_local, num_sites, device,
                           timeout_s) if use else None
    if not ctx.distributed:
        return ws
    mine = (ctx.role, ctx.tp_rank, ws.handle() if ws is not None else None, ws is not None)
    allh: list = [None] * ctx.world_size
    dist.all_gather_object(allh, mine, group=ctx.cpu_group)
    if ws is not None and ws.world > 1:
        group = {tp: (h, ok) for role, tp, h, ok in allh if role == ctx.role}
        if len(group) != ctx.tp_size or not all(ok for _, ok in group.values()):
            ws.close()
            ws = None
        else:
            ws.connect([group[r][0] for r in range(ctx.tp_size)])
    torch.cuda.synchronize(device)   # regions are zero before any peer may write them
    dist.barrier(group=ctx.cpu_group)
    return ws
