"""Standalone disaggregated prefill/decode engine (one process per GPU).

Request flow (every rank calls :meth:`PDEngine.generate` with the same
prompt, SPMD):

* prefill ranks run the prompt's first ``T-1`` tokens through the model; after
  each layer's K/V are written the fused encode kernel pushes the compressed
  frame of that layer into the paired decode rank's receive slot (NVLink peer
  stores) and publishes it — transfer overlaps the remaining layers;
* decode ranks launch one persistent fused decode that waits for each layer
  and writes the paged KV cache, then compute the last prompt token (as the
  reference's consumer does: it claims ``prompt_len - 1`` external tokens,
  kvserve_v1/connector/compressed_kv_connector.py:511-524) and continue with
  greedy decode steps replayed from one CUDA graph per step.

All timings are CUDA events on each rank's own streams relative to a start
event recorded right after a device-side NCCL barrier, so per-rank times are
aligned to within the barrier skew and the max over ranks is meaningful.
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass, field
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops
from ..models.config import ModelConfig
from ..models.llama import LlamaShard
from ..parallel.context import ParallelContext
from ..parallel.decode_allreduce import create_decode_collectives
from ..parallel.tp_allreduce import create_tp_allreduce
from ..transport.p2p import FrameReceiver, FrameSender
from ..utils.trace import decode_stamps, nvtx_range, summarize_stamps, trace_enabled, write_trace_row
from ..session.tp_plan import HeadCopy, head_shard, transfer_plan
from .kv_cache import PagedKVCache
from .transfer import KVTransfer, TransferProfile


@dataclass
class RequestTiming:
    """Milliseconds from the request start on this rank (NaN where n/a)."""
    prefill_done: float = float("nan")
    encode_start: float = float("nan")      # layer 0's encode may start (its K/V exist)
    encode_done: float = float("nan")
    ingest_done: float = float("nan")
    first_token: float = float("nan")
    all_done: float = float("nan")
    first_token_host: float = float("nan")   # wall ms from generate() entry to first token on the host
    request_host: float = float("nan")       # wall ms of the whole generate() call
    launches: int = 0                        # kernels of this package launched for the request
    payload_bytes: int = 0
    raw_bytes: int = 0
    trace: dict = field(default_factory=dict)  # device stamp summary (KVSERVE_TRACE=1)


@dataclass
class GenerateResult:
    tokens: Optional[list[int]]
    timing: RequestTiming


class PDEngine:
    def __init__(self, cfg: ModelConfig, ctx: ParallelContext, profile: TransferProfile, max_prompt: int = 8192,
                 max_new_tokens: int = 128, block_size: int = 16, seed: int = 0, link_gbps: float = 0.0,
                 use_graphs: bool = True, ingest_timeout_s: float = 30.0, encode_ctas: int = 222,
                 profiles: Optional[dict] = None, num_slots: int = 2, max_batch: int = 1,
                 checkpoint: Optional[str] = None):
        self.cfg, self.ctx, self.profile = cfg, ctx, profile
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.max_prompt, self.max_new, self.block_size = max_prompt, max_new_tokens, block_size
        self.use_graphs = use_graphs
        self.ingest_timeout_ns = int(ingest_timeout_s * 1e9)
        # CTAs of each layer's encode launches (KVSERVE_ENCODE_CTAS overrides):
        # fewer leave more SMs to the prefill's own kernels beside them
        self.encode_ctas = int(os.environ.get("KVSERVE_ENCODE_CTAS", encode_ctas))
        self.rate_bytes_per_ns = link_gbps / 8.0 if link_gbps else 0.0
        self.model = LlamaShard(cfg, ctx.tp_rank, ctx.tp_size, self.device, seed, ctx.tp_group,
                                max_position=max_prompt + max_new_tokens + block_size)
        m = self.model
        if checkpoint:          # weights saved by LlamaShard.save, one file per TP shard
            m.load(checkpoint)
        # prefill ranks reduce their row-parallel projections inside the GEMM
        m.tp_ar = create_tp_allreduce(ctx, max_prompt, cfg.hidden, self.device, participate=ctx.is_prefill)
        # decode ranks fuse their per-step collectives into the projections
        m.decode_coll = create_decode_collectives(ctx, cfg.hidden, m.vocab_local, m.decode_sites(), self.device,
                                                  participate=ctx.is_decode)
        # ---- KV hand-off plan: the KV-head ranges each prefill rank sends to
        # each decode rank (one full-shard copy per TP pair when both groups
        # have the same size; heterogeneous TP splits or merges the ranges,
        # session.tp_plan).  This rank's copies, in plan order:
        n_pre = ctx.num_prefill if ctx.distributed else 1
        n_dec = ctx.world_size - n_pre if ctx.distributed else 1
        self.plan = transfer_plan(n_pre, n_dec, cfg.num_kv_heads)
        if ctx.role == "decode":
            self.copies = [c for c in self.plan if c.dst_rank == ctx.tp_rank]
        else:
            self.copies = [c for c in self.plan if c.src_rank == ctx.tp_rank]
        # one transfer geometry per (selectable profile, copy) ("default" =
        # `profile`); the receive slots are sized for the largest frame
        self.xfer_sets = {name: [self._copy_transfer(p, c, n_pre, max_prompt) for c in self.copies]
                          for name, p in {"default": profile, **(profiles or {})}.items()}
        self.xfers = {name: xs[0] for name, xs in self.xfer_sets.items()}
        self.xfer = self.xfers["default"]
        self.compute = torch.cuda.current_stream(self.device)
        self.seq = 0
        self.status = ops.device_status(self.device)
        # %globaltimer stamps of the hand-off kernels (KVSERVE_TRACE=1)
        self.trace = torch.zeros((cfg.num_layers, 4), dtype=torch.int64, device=self.device) \
            if trace_enabled() else None
        self.d_first = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._tok_host = torch.empty(1, dtype=torch.int32, pin_memory=True)
        L = cfg.num_layers
        if ctx.is_prefill:
            self.k_buf = torch.empty((L, max_prompt, m.hkv, m.D), dtype=torch.bfloat16, device=self.device)
            self.v_buf = torch.empty_like(self.k_buf)
            self.enc_stream = torch.cuda.Stream(self.device, priority=-1)
            self.layer_events = [torch.cuda.Event() for _ in range(L)]
            self.pacing = torch.zeros(2, dtype=torch.int64, device=self.device)
            self.positions = torch.arange(max_prompt, dtype=torch.int32, device=self.device)
        if ctx.is_decode:
            self.max_blocks = (max_prompt + max_new_tokens + block_size - 1) // block_size + 1
            # room for `max_batch` requests of the largest size (continuous
            # batching, engine.pipeline) plus one scratch block for padding rows
            self.max_batch = max(1, int(max_batch))
            self.kv = PagedKVCache(L, self.max_batch * self.max_blocks + 1, block_size, m.hkv, m.D, self.device)
            self._scratch_block = self.kv.allocate(1)
            self.ingest_stream = torch.cuda.Stream(self.device, priority=-1)
            self._init_decode_buffers()
        # ---- channels: one receiver (decode side) per copy, with its slots,
        # flags and credits; the prefill side maps each of its copies' receivers
        self.receivers: list[FrameReceiver] = []
        self.senders: list[FrameSender] = []
        # receive slots of the channel; request `seq` uses slot seq % num_slots
        # and waits for the slot's credit from its previous request
        self.num_slots = max(1, int(num_slots))
        self._slot_seq = [0] * self.num_slots
        if ctx.is_decode:
            for i in range(len(self.copies)):
                stride = max(xs[i].frame_stride for xs in self.xfer_sets.values())
                self.receivers.append(FrameReceiver(L, stride, self.num_slots, self.device))
        if not ctx.distributed:
            self.senders = [FrameSender(local=r, device=self.device) for r in self.receivers]
        else:
            local = [r.handles() for r in self.receivers] if ctx.role == "decode" else None
            allh = [None] * ctx.world_size
            dist.all_gather_object(allh, local, group=ctx.cpu_group)
            if ctx.role == "prefill":
                for c in self.copies:
                    theirs = [x for x in self.plan if x.dst_rank == c.dst_rank]
                    self.senders.append(FrameSender(handles=allh[n_pre + c.dst_rank][theirs.index(c)],
                                                    device=self.device))
            dist.barrier(group=ctx.cpu_group)
            self._barrier_t = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.receiver: Optional[FrameReceiver] = self.receivers[0] if self.receivers else None
        self.sender: Optional[FrameSender] = self.senders[0] if self.senders else None
        self._graph: Optional[torch.cuda.CUDAGraph] = None
        torch.cuda.synchronize(self.device)

    def _copy_transfer(self, profile: TransferProfile, c: HeadCopy, n_pre: int, max_prompt: int) -> KVTransfer:
        """Transfer geometry of one copy: its heads as an aligned slice of the
        model's KV heads (the slice index and count play the TP rank/size)."""
        cfg = self.cfg
        first = head_shard(c.src_rank, n_pre, cfg.num_kv_heads).first + c.src_head
        if cfg.num_kv_heads % c.heads or first % c.heads:
            raise ValueError("KV-head copies must be aligned slices of the model's KV heads")
        return KVTransfer(profile, cfg.num_layers, cfg.num_kv_heads, c.heads, self.model.D, first // c.heads,
                          cfg.num_kv_heads // c.heads, self.device, self.max_prompt, cfg.score_model_name)

    # ------------------------------------------------- hand-off per copy
    def _cache_view(self, c: HeadCopy) -> torch.Tensor:
        """The paged cache restricted to the copy's KV heads (a strided view)."""
        if c.dst_head == 0 and c.heads == self.model.hkv:
            return self.kv.cache
        return self.kv.cache[:, :, :, :, c.dst_head:c.dst_head + c.heads]

    def _encode_layer(self, l: int, T: int, slot: int, seq: int, name: str, rate: float,
                      table: Optional[torch.Tensor] = None) -> None:
        """Encode + push layer ``l`` of every copy of this prefill rank (on the
        current stream); colocated, decode it into the paged cache too."""
        dist_ = self.ctx.distributed
        for i, (c, x, snd) in enumerate(zip(self.copies, self.xfer_sets[name], self.senders)):
            hs = slice(c.src_head, c.src_head + c.heads)
            tr = self.trace if i == 0 else None
            x.encode(l, self.k_buf[l, :T, hs], self.v_buf[l, :T, hs], snd.frame_ptr(slot, l),
                     snd.flag_ptr(slot, l) if dist_ else 0, seq, self.pacing, rate, self.encode_ctas, trace=tr)
            if not dist_:
                x.ingest_layer(l, T, snd.frame_ptr(slot, l), self._cache_view(c), table, self.status, seq, trace=tr)

    def _ingest_all(self, T: int, slot: int, seq: int, name: str, table: torch.Tensor, max_ctas: int = 148) -> None:
        """Decode every copy of this decode rank into its heads of the paged
        cache (on the current stream; each kernel waits on its layer flags)."""
        for i, (c, x, r) in enumerate(zip(self.copies, self.xfer_sets[name], self.receivers)):
            x.ingest_all(T, r.slot_base(slot), r.frame_stride, r.flags_base(slot), self._cache_view(c), table,
                         self.status, seq, self.ingest_timeout_ns, max_ctas=max_ctas,
                         trace=self.trace if i == 0 else None)

    def request_bytes(self, T: int, name: str = "default") -> tuple[int, int]:
        """(payload, raw) bytes of this rank's copies of one T-token request."""
        xs = self.xfer_sets[name]
        return sum(x.payload_bytes(T) for x in xs), sum(x.raw_bytes(T) for x in xs)

    # ----------------------------------------------------------- decode state
    def _init_decode_buffers(self) -> None:
        dev = self.device
        self.d_ids = torch.zeros(1, dtype=torch.int32, device=dev)
        self.d_pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.d_ctx = torch.ones(1, dtype=torch.int32, device=dev)
        self.d_slot = torch.zeros(1, dtype=torch.int32, device=dev)
        self.d_step = torch.zeros(1, dtype=torch.int32, device=dev)
        self.d_table = torch.zeros((1, self.max_blocks), dtype=torch.int32, device=dev)
        self.d_out = torch.zeros(self.max_new + 1, dtype=torch.int32, device=dev)
        self.d_init_host = torch.zeros(5 + self.max_blocks, dtype=torch.int32).pin_memory()
        self.d_init_dev = torch.zeros(5 + self.max_blocks, dtype=torch.int32, device=dev)
        hq, D = self.model.hq, self.model.D
        splits = ops.ext().paged_decode_splits(1, self.model.hkv, self.max_prompt + self.max_new)
        self.attn_scratch = (torch.empty(hq * splits * D, dtype=torch.float32, device=dev),
                             torch.empty(hq * splits * 2, dtype=torch.float32, device=dev))

    def _first_host(self, tok: torch.Tensor, ev: dict, timing: "RequestTiming", t_host0: float) -> None:
        """Record the first-token event and stream the token to the host (what
        a server returns first)."""
        ev["first"].record(self.compute)
        self._tok_host.copy_(tok[:1], non_blocking=True)
        done = torch.cuda.Event()
        done.record(self.compute)
        done.synchronize()
        timing.first_token_host = 1e3 * (time.perf_counter() - t_host0)

    def _decode_step(self) -> None:
        tok = self.model.decode_step(self.d_ids, self.d_pos, self.d_slot, self.kv.cache, self.d_table, self.d_ctx,
                                     self.max_prompt + self.max_new, attn_scratch=self.attn_scratch)
        ops.count_launches(1)
        ops.ext().decode_advance(tok, self.d_ids, self.d_pos, self.d_ctx, self.d_slot, self.d_table,
                                 self.block_size, self.d_out, self.d_step)

    def _load_decode_state(self, first_token_id: int, position: int, blocks: list[int]) -> None:
        h = self.d_init_host
        bs = self.block_size
        h.zero_()
        h[0] = first_token_id
        h[1] = position
        h[2] = position + 1
        h[3] = blocks[position // bs] * bs + position % bs
        h[4] = 1  # d_out[0] holds the first token (sampled by the prefill)
        h[5:5 + len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
        self.d_init_dev.copy_(h, non_blocking=True)
        d = self.d_init_dev
        self.d_ids.copy_(d[0:1])
        self.d_pos.copy_(d[1:2])
        self.d_ctx.copy_(d[2:3])
        self.d_slot.copy_(d[3:4])
        self.d_step.copy_(d[4:5])
        self.d_table[0].copy_(d[5:])

    def _ensure_graph(self) -> None:
        if not self.use_graphs or self._graph is not None:
            return
        # warm up on the scratch block, then capture one step
        self._load_decode_state(0, 0, self._scratch_block * self.max_blocks)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(self.compute)
        with torch.cuda.stream(s):
            for _ in range(2):
                self._load_decode_state(0, 0, self._scratch_block * self.max_blocks)
                self._decode_step()
        self.compute.wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        self._load_decode_state(0, 0, self._scratch_block * self.max_blocks)
        torch.cuda.synchronize(self.device)
        c0 = ops.launches()
        with torch.cuda.graph(g, stream=s):
            self._decode_step()
        torch.cuda.synchronize(self.device)
        self._graph_launches = ops.launches() - c0
        self._graph = g

    def warmup(self, prompt_len: int = 256) -> None:
        """Compile-free warm-up: runs one short request through every path."""
        if self.ctx.is_decode:
            self._ensure_graph()
        ids = torch.randint(0, self.cfg.vocab, (prompt_len,), dtype=torch.int32)
        self.generate(ids, 2)

    # --------------------------------------------------------------- request
    def _barrier(self) -> None:
        """Device-side barrier: every rank's stream waits for all ranks."""
        if self.ctx.distributed:
            dist.all_reduce(self._barrier_t, group=self.ctx.world_group)

    def _host_barrier(self) -> None:
        """Host-side barrier: returns once every rank's host has reached it
        (so no rank is still finishing an earlier request)."""
        if self.ctx.distributed:
            dist.barrier(group=self.ctx.cpu_group)

    # ------------------------------------------------- slots and credits
    def _next_seq(self) -> tuple[int, int]:
        """(sequence number, receive slot) of the next request."""
        self.seq += 1
        return self.seq, self.seq % self.num_slots

    def _take_credit(self, slot: int, seq: int) -> None:
        """Producer, on the current stream before the slot's first store:
        acquire-wait (bounded) until every decode rank this rank feeds has
        read the slot's previous request out of it."""
        prev = self._slot_seq[slot]
        self._slot_seq[slot] = seq
        if self.ctx.distributed and prev:
            for snd in self.senders:
                ops.count_launches(1)
                ops.ext().wait_flag(snd.credit_ptr(slot), prev, self.ingest_timeout_ns, self.status)

    def check_slots(self) -> None:
        """With ``KVSERVE_SLOT_CANARIES=1``: fail if a producer wrote past a
        receive slot into its guard region (no-op without guards)."""
        for i, r in enumerate(self.receivers):
            bad = r.damaged_slots()
            if bad:
                raise RuntimeError(f"KV hand-off: receive channel {i} slot(s) {bad} overran into their guard "
                                   f"region (frame layout mismatch between the peers?)")

    def _return_credit(self, slot: int, seq: int) -> None:
        """Consumer, on the stream of the last kernel that read the slot."""
        self._slot_seq[slot] = seq
        if self.ctx.distributed:
            for r in self.receivers:
                ops.count_launches(1)
                ops.ext().store_release_u32(r.credit_ptr(slot), seq)

    def _publish_token(self, first: torch.Tensor, slot: int, seq: int) -> None:
        """Prefill side: the sampled first token next to the flags of every
        receiver this rank feeds."""
        for snd in self.senders:
            ops.count_launches(1)
            ops.ext().publish_token(first, snd.token_ptr(slot), seq)

    def _take_token(self, slot: int, seq: int, out: torch.Tensor, out2: Optional[torch.Tensor] = None) -> None:
        ops.count_launches(1)
        ops.ext().take_token(self.receivers[0].token_ptr(slot), seq, self.ingest_timeout_ns, out, out2, self.status)

    def _launch_prefill(self, ids: torch.Tensor, seq: int, slot: int, xfer: str, rate: float,
                        ev: Optional[dict] = None, table: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Prefill side of one request (asynchronous): the prompt's forward
        pass with each layer's K/V encoded and pushed into receive slot
        ``slot`` on the encode stream right after the layer is written (after
        the slot's credit is taken), and the sampled first token published
        next to the slot's flags.  Colocated, each layer is also decoded into
        the paged cache (``table``) on the encode stream.  Returns the first
        token (int32 [1] on the device)."""
        ctx, m = self.ctx, self.model
        T = int(ids.numel())
        enc = self.enc_stream
        enc.wait_stream(self.compute)
        with torch.cuda.stream(enc):
            self._take_credit(slot, seq)

        def hook(l: int) -> None:
            self.layer_events[l].record(self.compute)
            enc.wait_event(self.layer_events[l])
            if l == 0 and ev is not None:
                ev["enc_start"].record(enc)
            with torch.cuda.stream(enc), nvtx_range(f"kv encode L{l}"):
                self._encode_layer(l, T, slot, seq, xfer, rate, table)

        first = m.prefill(ids, self.positions[:T], self.k_buf, self.v_buf, layer_hook=hook, sample=True)
        if ev is not None:
            ev["prefill"].record(self.compute)
        if ctx.distributed:
            # the token lands next to the layer flags of the decode slots
            self._publish_token(first, slot, seq)
        if ev is not None:
            ev["encode"].record(enc)
        return first

    def generate(self, prompt_ids: torch.Tensor, max_new_tokens: Optional[int] = None,
                 return_tokens: bool = True, sync: bool = True, profile: Optional[str] = None,
                 link_gbps: Optional[float] = None) -> GenerateResult:
        """Serve one request.  ``prompt_ids`` is a host int32 tensor (pinned
        preferably); the prompt is copied to the device inside the request.
        ``profile`` names one of the engine's transfer profiles (every rank
        must pass the same name); ``link_gbps`` paces this request's KV
        stores at that rate (an emulated link cap; None keeps the engine's).

        ``sync`` aligns all ranks on a host collective before the request so
        per-request device timings share a start; with ``sync=False`` a decode
        rank relies on the per-layer frame flags alone (a prefill rank that
        never publishes then surfaces as a device-side timeout status)."""
        ctx, m = self.ctx, self.model
        if sync:
            # the request starts once every rank is free for it: the host clock
            # must not charge the previous request's decode to this TTFT
            self._host_barrier()
        t_host0 = time.perf_counter()
        if profile is not None and profile not in self.xfers:
            raise KeyError(f"unknown transfer profile {profile!r}; have {sorted(self.xfers)}")
        xfer = profile or "default"
        rate = self.rate_bytes_per_ns if link_gbps is None else (link_gbps / 8.0 if link_gbps else 0.0)
        n_new = self.max_new if max_new_tokens is None else max_new_tokens
        if n_new < 1 or n_new > self.max_new:
            raise ValueError(f"max_new_tokens must be in [1, {self.max_new}]")
        T = int(prompt_ids.numel())
        if T < 1 or T > self.max_prompt:
            raise ValueError(f"prompt length must be in [1, {self.max_prompt}]")
        # The prefill covers the whole prompt and samples the first token; the
        # KV of all T tokens is handed to the decode side with that token.
        Tx = T
        seq, slot = self._next_seq()
        ev = {k: torch.cuda.Event(enable_timing=True)
              for k in ("start", "prefill", "enc_start", "encode", "ingest", "first", "end")}
        if sync:
            self._barrier()
        c_launch0 = ops.launches()
        replays = 0
        ev["start"].record(self.compute)
        if self.trace is not None:
            self.trace.zero_()
        ids = prompt_ids.to(self.device, non_blocking=True)
        pay, raw = self.request_bytes(Tx, xfer)
        timing = RequestTiming(payload_bytes=pay, raw_bytes=raw)
        blocks = table = None
        if ctx.is_decode:
            blocks = self.kv.allocate(T + n_new)
            table = self.kv.block_table(blocks, self.max_blocks)
            if ctx.distributed:
                self.ingest_stream.wait_stream(self.compute)
                with torch.cuda.stream(self.ingest_stream), nvtx_range("kv ingest"):
                    self._ingest_all(Tx, slot, seq, xfer, table)
                    ev["ingest"].record(self.ingest_stream)
        if ctx.is_prefill:
            first = self._launch_prefill(ids[:Tx], seq, slot, xfer, rate, ev, table)
            if not ctx.distributed:
                ev["ingest"].record(self.enc_stream)
                self.d_first.copy_(first)
            else:
                self._first_host(first, ev, timing, t_host0)
        tokens = None
        if ctx.is_decode:
            self.compute.wait_event(ev["ingest"])
            self._ensure_graph()
            self._load_decode_state(0, T, blocks)
            if ctx.distributed:
                self._take_token(slot, seq, self.d_ids, self.d_out)
                self._return_credit(slot, seq)
            else:
                self.d_ids.copy_(self.d_first)
                self.d_out[0:1].copy_(self.d_first)
            self._first_host(self.d_ids, ev, timing, t_host0)
            for _ in range(n_new - 1):
                if self._graph is not None:
                    self._graph.replay()
                    replays += 1
                else:
                    self._decode_step()
            out_host = torch.empty(n_new, dtype=torch.int32, pin_memory=True)
            out_host.copy_(self.d_out[:n_new], non_blocking=True)
            ev["end"].record(self.compute)
            torch.cuda.synchronize(self.device)
            tokens = out_host.tolist() if return_tokens else None
            self.kv.release(blocks)
        else:
            ev["end"].record(self.compute)
            torch.cuda.synchronize(self.device)
        st = int(self.status[0].item())
        if st != 0:
            self.status.zero_()
            raise RuntimeError(f"KV hand-off failed on rank {ctx.rank}: {ops.STATUS_NAMES.get(st, st)}")
        self.check_slots()
        dc = m.decode_coll
        if dc is not None and int(dc.status[0].item()) != 0:
            code = int(dc.status[0].item())
            dc.status.zero_()
            raise RuntimeError(f"decode collective failed on rank {ctx.rank}: status {code} (peer timeout)")
        if self.trace is not None:
            st_ = decode_stamps(self.trace.cpu())
            timing.trace = summarize_stamps(st_)
            write_trace_row({"rank": ctx.rank, "role": ctx.role, "seq": seq, "tokens": T,
                             "payload_bytes": timing.payload_bytes, **timing.trace, **st_})
        timing.launches = ops.launches() - c_launch0 + replays * getattr(self, "_graph_launches", 0)
        timing.request_host = 1e3 * (time.perf_counter() - t_host0)
        e = lambda k: ev["start"].elapsed_time(ev[k])  # noqa: E731
        timing.first_token = e("first")
        if ctx.is_prefill:
            timing.prefill_done = e("prefill")
            timing.encode_start = e("enc_start")
            timing.encode_done = e("encode")
        if ctx.is_decode:
            timing.ingest_done = e("ingest")
            timing.all_done = e("end")
        return GenerateResult(tokens, timing)

    def measure_handoff(self, T: int, profile: Optional[str] = None) -> dict:
        """Device time of one request's whole KV hand-off on its own: every
        layer of the last prompt's K/V (still in the prefill buffers) encoded
        and pushed back to back, and decoded into the paged cache, without a
        prefill running beside it.  This is the per-request KV-transfer time
        of the transfer path alone (the reference's connector does the same
        work after its prefill, kvserve_v1/connector/compressed_kv_connector.py:393-497
        and :235-372).  Milliseconds from a common device start: ``encode_ms``
        (prefill side: last frame published) and ``ingest_ms`` (decode side:
        last layer written), NaN where the rank has no such part."""
        ctx = self.ctx
        xfer = profile or "default"
        if T < 1 or T > self.max_prompt:
            raise ValueError(f"T must be in [1, {self.max_prompt}]")
        self._host_barrier()
        seq, slot = self._next_seq()
        start, enc_end, ing_end = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        self._barrier()
        start.record(self.compute)
        blocks = table = None
        if ctx.is_decode:
            blocks = self.kv.allocate(T)
            table = self.kv.block_table(blocks, self.max_blocks)
            if ctx.distributed:
                self.ingest_stream.wait_stream(self.compute)
                with torch.cuda.stream(self.ingest_stream):
                    self._ingest_all(T, slot, seq, xfer, table)
                    ing_end.record(self.ingest_stream)
                    self._return_credit(slot, seq)
        if ctx.is_prefill:
            enc = self.enc_stream
            enc.wait_stream(self.compute)
            with torch.cuda.stream(enc):
                self._take_credit(slot, seq)
                for l in range(self.cfg.num_layers):
                    self._encode_layer(l, T, slot, seq, xfer, 0.0, table)
                enc_end.record(enc)
                if not ctx.distributed:
                    ing_end.record(enc)
        torch.cuda.synchronize(self.device)
        if blocks is not None:
            self.kv.release(blocks)
        st = int(self.status[0].item())
        if st != 0:
            self.status.zero_()
            raise RuntimeError(f"KV hand-off failed on rank {ctx.rank}: {ops.STATUS_NAMES.get(st, st)}")
        self.check_slots()
        nan = float("nan")
        return {"encode_ms": start.elapsed_time(enc_end) if ctx.is_prefill else nan,
                "ingest_ms": start.elapsed_time(ing_end) if ctx.is_decode else nan,
                "payload_bytes": self.request_bytes(T, xfer)[0], "raw_bytes": self.request_bytes(T, xfer)[1]}

    def decode_kernel_table(self, prompt_ids: torch.Tensor, steps: int = 8) -> list:
        """Per-kernel device time of this rank's decode steps, taken with the
        PyTorch profiler (CUPTI) around ``steps`` graph replays after one
        request's prefill and hand-off: ``[(kernel, calls_per_step,
        us_per_step)]`` sorted by time.  Evidence of where a decode step goes,
        not a timing of record (a profiler adds overhead).  Every rank calls
        it (it serves one request)."""
        from torch.profiler import ProfilerActivity, profile
        res = self.generate(prompt_ids, min(self.max_new, steps + 1))
        table = []
        if self.ctx.is_decode and self._graph is not None:
            torch.cuda.synchronize(self.device)
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                for _ in range(steps):
                    self._graph.replay()
                torch.cuda.synchronize(self.device)
            for ev in prof.key_averages():
                t = getattr(ev, "device_time_total", None) or getattr(ev, "cuda_time_total", 0)
                if t and ev.count:
                    table.append((ev.key[:90], round(ev.count / steps, 2), round(t / steps, 2)))
            table.sort(key=lambda r: -r[2])
        del res
        return table

    def prefill_kernel_table(self, prompt_ids: torch.Tensor, top: int = 24) -> list:
        """Per-kernel device time of one request on this rank, taken with the
        PyTorch profiler (CUPTI) around the whole request (prefill, hand-off
        and one decode step): ``[(kernel, calls, us)]`` sorted by time.  On a
        prefill rank this is the prefill's breakdown (GEMMs, attention,
        norms, encode); on a decode rank the ingest and the step.  Evidence,
        not a timing of record.  Every rank calls it (it serves one request)
        and every rank profiles, so the ranks stay in step."""
        from torch.profiler import ProfilerActivity, profile
        torch.cuda.synchronize(self.device)
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            if self.ctx.distributed:
                # the profiler's start-up time differs per rank: line up first
                import torch.distributed as dist
                dist.barrier(group=self.ctx.cpu_group)
            res = self.generate(prompt_ids, min(self.max_new, 2))
            torch.cuda.synchronize(self.device)
        table = []
        for ev in prof.key_averages():
            t = getattr(ev, "device_time_total", None) or getattr(ev, "cuda_time_total", 0)
            if t and ev.count:
                table.append((ev.key[:90], int(ev.count), round(float(t), 1)))
        table.sort(key=lambda r: -r[2])
        del res
        return table[:top]

    def close(self) -> None:
        self._graph = None
        if self.model.decode_coll is not None:
            torch.cuda.synchronize(self.device)
            self.model.decode_coll.close()
            self.model.decode_coll = None
        if self.model.tp_ar is not None:
            torch.cuda.synchronize(self.device)
            self.model.tp_ar.close()
            self.model.tp_ar = None
        for snd in self.senders:
            snd.close()
        if self.receivers:
            torch.cuda.synchronize(self.device)
        for r in self.receivers:
            r.close()
