"""Pipelined PD serving: prefill of request i+1 overlaps decode of request i.

:meth:`PDEngine.generate` serves one request at a time behind a host
barrier.  This module drives the same engine as a server:

* prefill ranks take requests in arrival order (a shared wall clock; the
  schedule is known to every rank), run each prompt's forward pass with the
  per-layer fused encode + NVLink push into receive slot ``seq % num_slots``
  and go on with the next request at once — the encode kernels take the
  slot's device credit first (bounded acquire wait), so the prefill side runs
  at most ``num_slots`` requests ahead of the decode side's ingest;
* decode ranks run **continuous batching**: a batch of up to ``max_batch``
  rows (requests) advances one token per step from CUDA graphs captured for
  1, 2, 4 and 8 rows; a request joins the batch as soon as its KV has been
  ingested into the paged cache (fused decode kernel on a side stream,
  concurrent with the batch's steps, limited to a few CTAs) and leaves when
  its tokens are done, and the slot's credit is returned right after the
  ingest kernel has read it.

Control plane: the job's c10d store (keys under a per-run prefix) carries
"request i launched" from the prefill leader and "request i ingested" from
the decode leader, plus the leader's profile decision for each request; the
decode TP ranks follow their leader's per-iteration action (a small gloo
broadcast) so that every rank replays the same graph with the same rows —
the fused decode collectives pair them step by step.

The reference's connector moves one request's KV per vLLM scheduler step
(kvserve_v1/connector/compressed_kv_connector.py:393-497) with receive
credits in its NCCL transport (kvserve_v1/transport/nccl_transport.py:519-560)
and a per-slot state machine in the Mooncake variant
(kvsfuse-vllm0.30.0/mooncake/compression/state.py:14-72); here the credits
live in the decode GPU's memory and are taken by the producer's kernels.
"""
from __future__ import annotations

import json
import os
import time
from collections import deque
from dataclasses import dataclass, field
from typing import Callable, Optional

import torch
import torch.distributed as dist

from .. import ops

BUCKETS = (1, 2, 4, 8)
# state fields of a batch row (field-major [F, rows] int32 device tensor)
F_IDS, F_POS, F_CTX, F_SLOT, F_STEPS, F_ACTIVE = range(6)
NUM_FIELDS = 6


@dataclass
class Request:
    index: int
    prompt: torch.Tensor              # host int32 [T] (pinned preferably)
    max_new: int
    arrival_s: float = 0.0            # seconds after the run's common start
    profile: Optional[str] = None     # engine transfer profile (None: the default)
    link_gbps: Optional[float] = None


@dataclass
class RequestRecord:
    """Host wall-clock milliseconds after the request's arrival (NaN where
    this rank has no such event)."""
    index: int
    arrival_ms: float
    profile: str = "default"
    launch_ms: float = float("nan")        # prefill launched (prefill ranks)
    prefill_ms: float = float("nan")       # prefill done, first token published (prefill ranks)
    kv_ready_ms: float = float("nan")      # KV in the paged cache (decode ranks)
    first_token_ms: float = float("nan")   # first token on the decode host (= TTFT)
    done_ms: float = float("nan")          # all tokens on the decode host
    tokens: Optional[list] = None
    extra: dict = field(default_factory=dict)


def bucket_for(n: int) -> int:
    for b in BUCKETS:
        if n <= b:
            return b
    raise ValueError(f"batch of {n} rows exceeds {BUCKETS[-1]}")


class BatchDecoder:
    """Continuous-batching decode state of one decode rank: ``rows`` batch
    rows over the engine's paged cache, one CUDA graph per bucket size."""

    def __init__(self, engine, rows: int):
        if rows > BUCKETS[-1] or rows > engine.max_batch:
            raise ValueError(f"rows must be <= {BUCKETS[-1]} and <= the engine's max_batch ({engine.max_batch})")
        self.eng = engine
        self.rows = rows
        dev = engine.device
        self.max_new = engine.max_new
        self.max_ctx = engine.max_prompt + engine.max_new
        self.scratch_block = engine._scratch_block[0]
        bs = engine.block_size
        self.state = torch.zeros((NUM_FIELDS, rows), dtype=torch.int32, device=dev)
        self.table = torch.full((rows, engine.max_blocks), self.scratch_block, dtype=torch.int32, device=dev)
        self.out = torch.zeros((rows, self.max_new + 1), dtype=torch.int32, device=dev)
        self.pad_col = torch.tensor([0, 0, 1, self.scratch_block * bs, 0, 0], dtype=torch.int32, device=dev)
        for r in range(rows):
            self.state[:, r].copy_(self.pad_col)
        # a small ring of pinned staging rows: a row is rewritten only after
        # the copy that last read it has completed
        self.row_host = [torch.zeros(NUM_FIELDS + engine.max_blocks, dtype=torch.int32).pin_memory()
                         for _ in range(4)]
        self.row_ev: list[Optional[torch.cuda.Event]] = [None] * 4
        self._ring = 0
        self.row_dev = torch.zeros(NUM_FIELDS + engine.max_blocks, dtype=torch.int32, device=dev)
        m = engine.model
        splits = max(ops.ext().paged_decode_splits(b, m.hkv, self.max_ctx) * b for b in BUCKETS if b <= rows)
        self.attn_scratch = (torch.empty(m.hq * splits * m.D, dtype=torch.float32, device=dev),
                             torch.empty(m.hq * splits * 2, dtype=torch.float32, device=dev))
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.graph_launches: dict[int, int] = {}

    # ------------------------------------------------------------- steps
    def _step(self, b: int) -> None:
        st, eng = self.state, self.eng
        tok = eng.model.decode_step(st[F_IDS, :b], st[F_POS, :b], st[F_SLOT, :b], eng.kv.cache, self.table[:b],
                                    st[F_CTX, :b], self.max_ctx, attn_scratch=self.attn_scratch)
        ops.count_launches(1)
        ops.ext().batch_advance(tok, st[F_ACTIVE, :b], st[F_IDS, :b], st[F_POS, :b], st[F_CTX, :b],
                                st[F_SLOT, :b], self.table[:b], eng.block_size, self.out[:b], st[F_STEPS, :b])

    def capture(self) -> None:
        """One graph per bucket (all rows padding while capturing)."""
        eng = self.eng
        s = torch.cuda.Stream(eng.device)
        s.wait_stream(eng.compute)
        for b in BUCKETS:
            if b > self.rows:
                break
            with torch.cuda.stream(s):
                for _ in range(2):
                    self._step(b)
            torch.cuda.synchronize(eng.device)
            g = torch.cuda.CUDAGraph()
            c0 = ops.launches()
            with torch.cuda.graph(g, stream=s):
                self._step(b)
            torch.cuda.synchronize(eng.device)
            self.graph_launches[b] = ops.launches() - c0
            self.graphs[b] = g
        eng.compute.wait_stream(s)

    def step(self, active: int) -> int:
        """Advance rows [0, active) by one token (padding rows up to the
        bucket size ride along inactive); returns the launches it replayed."""
        b = bucket_for(active)
        self.graphs[b].replay()
        return self.graph_launches[b]

    # -------------------------------------------------------- join / leave
    def join(self, row: int, token_dev: torch.Tensor, position: int, blocks: list) -> None:
        """Row ``row`` starts a request whose prompt occupies positions
        [0, position) of ``blocks`` and whose first token (sampled by the
        prefill) is ``token_dev`` (int32 [1] on the device).  Ordered on the
        current stream."""
        bs = self.eng.block_size
        k = self._ring
        self._ring = (k + 1) % len(self.row_host)
        if self.row_ev[k] is not None:
            self.row_ev[k].synchronize()
        h = self.row_host[k]
        h.zero_()
        h[F_POS] = position
        h[F_CTX] = position + 1
        h[F_SLOT] = blocks[position // bs] * bs + position % bs
        h[F_STEPS] = 1
        h[F_ACTIVE] = 1
        h[NUM_FIELDS:NUM_FIELDS + len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
        self.row_dev.copy_(h, non_blocking=True)
        self.row_ev[k] = torch.cuda.Event()
        self.row_ev[k].record()
        self.state[:, row].copy_(self.row_dev[:NUM_FIELDS])
        self.state[F_IDS, row:row + 1].copy_(token_dev)
        self.table[row].copy_(self.row_dev[NUM_FIELDS:])
        self.out[row, 0:1].copy_(token_dev)

    def move(self, src: int, dst: int) -> None:
        self.state[:, dst].copy_(self.state[:, src])
        self.table[dst].copy_(self.table[src])
        self.out[dst].copy_(self.out[src])

    def clear(self, row: int) -> None:
        self.state[:, row].copy_(self.pad_col)
        self.table[row].fill_(self.scratch_block)


class PipelinedServer:
    """Serves a request schedule on a :class:`PDEngine` with prefill and
    decode overlapped.  Every rank constructs it (collective: it creates the
    role groups) and calls :meth:`serve` with the same schedule.  Colocated
    (one GPU) engines are not supported: their prefill and decode share one
    stream of work."""

    _runs = 0

    def __init__(self, engine, max_batch: int = 8, ingest_ctas: int = 32, poll_s: float = 2e-4,
                 timeout_s: float = 600.0):
        ctx = engine.ctx
        if not ctx.distributed:
            raise ValueError("pipelined serving needs separate prefill and decode ranks")
        self.eng, self.ctx = engine, ctx
        self.max_batch = max_batch
        self.ingest_ctas = ingest_ctas
        self.poll_s = poll_s
        self.timeout_s = timeout_s
        self.store = dist.distributed_c10d._get_default_store()
        # the role's gloo group of this replica (created by init_parallel)
        # and the role leader's global rank
        if ctx.role_cpu_groups is None:
            raise ValueError("the parallel context has no role groups (use parallel.context.init_parallel)")
        self.dec_group = ctx.role_cpu_groups["decode"]
        self.leader = ctx.global_ranks("prefill" if ctx.is_prefill else "decode")[0]
        self.decoder: Optional[BatchDecoder] = None
        if ctx.is_decode:
            self.decoder = BatchDecoder(engine, max_batch)
            self.decoder.capture()
        torch.cuda.synchronize(engine.device)
        dist.barrier(group=ctx.cpu_group)

    # ----------------------------------------------------------- helpers
    def _key(self, *parts) -> str:
        return "/".join(["kvs_pipe", str(self.ctx.replica), str(self._run)] + [str(p) for p in parts])

    def _wait_key(self, key: str) -> str:
        deadline = time.monotonic() + self.timeout_s
        while not self.store.check([key]):
            if time.monotonic() > deadline:
                raise TimeoutError(f"control-plane key {key!r} never arrived")
            time.sleep(self.poll_s)
        return self.store.get(key).decode()

    def _now_ms(self) -> float:
        return 1e3 * (time.time() - self.t0)

    # ------------------------------------------------------------- serve
    def serve(self, requests: list, decide: Optional[Callable] = None,
              feedback: Optional[Callable] = None) -> list:
        """Serve ``requests`` (:class:`Request`, arrival order).  ``decide(req,
        state)`` (prefill leader) may return a profile name per request;
        ``feedback(req, kv_ready_ms)`` receives the decode leader's KV-ready
        time of each ingested request before later decisions.  Returns this
        rank's :class:`RequestRecord` list; :func:`merge_records` combines
        them over ranks."""
        PipelinedServer._runs += 1
        self._run = PipelinedServer._runs
        ctx = self.ctx
        t0 = torch.tensor([time.time() + 0.2], dtype=torch.float64)
        dist.broadcast(t0, src=ctx.rank_offset, group=ctx.cpu_group)
        self.t0 = float(t0.item())
        recs = [RequestRecord(r.index, 1e3 * r.arrival_s) for r in requests]
        if ctx.is_prefill:
            self._serve_prefill(requests, recs, decide, feedback)
        else:
            self._serve_decode(requests, recs)
        torch.cuda.synchronize(self.eng.device)
        st = int(self.eng.status[0].item())
        if st != 0:
            self.eng.status.zero_()
            raise RuntimeError(f"pipelined serving failed on rank {ctx.rank}: {ops.STATUS_NAMES.get(st, st)}")
        dist.barrier(group=ctx.cpu_group)
        self.eng.check_slots()
        return recs

    # ------------------------------------------------------ prefill side
    def _serve_prefill(self, requests, recs, decide, feedback) -> None:
        eng, ctx = self.eng, self.ctx
        lead = ctx.global_rank == self.leader
        S = eng.num_slots
        fed = 0
        inflight: deque = deque()   # (index, compute-stream event, encode-stream event)

        def drain(block: bool) -> None:
            while inflight:
                i, e1, e2 = inflight[0]
                if block:
                    e1.synchronize()
                    e2.synchronize()
                elif not (e1.query() and e2.query()):
                    return
                recs[i].prefill_ms = self._now_ms() - recs[i].arrival_ms
                inflight.popleft()
                block = False

        state = {"prefill_ms": []}
        for i, req in enumerate(requests):
            while True:
                left = self.t0 + req.arrival_s - time.time()
                if left <= 0:
                    break
                drain(False)
                time.sleep(min(left, self.poll_s * 10))
            if lead and feedback is not None:
                while fed < i and self.store.check([self._key("ingested", fed)]):
                    info = json.loads(self.store.get(self._key("ingested", fed)).decode())
                    feedback(requests[fed], info["kv_ready_ms"])
                    fed += 1
            if lead:
                prof = (decide(req, state) if decide is not None else None) or req.profile or "default"
                self.store.set(self._key("decision", i), prof)
            else:
                prof = self._wait_key(self._key("decision", i))
            recs[i].profile = prof
            if i >= S:
                # host view of the slot's credit: the decode side has ingested
                # the slot's previous request (the device credit wait is then short)
                self._wait_key(self._key("ingested", i - S))
            seq, slot = eng._next_seq()
            rate = eng.rate_bytes_per_ns if req.link_gbps is None else (req.link_gbps / 8.0 if req.link_gbps else 0.0)
            ids = req.prompt.to(eng.device, non_blocking=True)
            # this forward pass overwrites the K/V buffers the previous request's encodes read
            eng.compute.wait_stream(eng.enc_stream)
            recs[i].launch_ms = self._now_ms() - recs[i].arrival_ms
            eng._launch_prefill(ids, seq, slot, prof, rate)
            e1, e2 = torch.cuda.Event(), torch.cuda.Event()
            e1.record(eng.compute)
            e2.record(eng.enc_stream)
            if lead:
                self.store.set(self._key("launched", i), json.dumps({"seq": seq, "slot": slot}))
            inflight.append((i, e1, e2))
            while len(inflight) > 1:   # at most one request queued behind the running one
                drain(True)
            done = [r.prefill_ms - r.launch_ms for r in recs[:i + 1] if r.prefill_ms == r.prefill_ms]
            state["prefill_ms"] = done
        drain(True)
        while inflight:
            drain(True)

    # ------------------------------------------------------- decode side
    def _serve_decode(self, requests, recs) -> None:
        eng, ctx, dec = self.eng, self.ctx, self.decoder
        lead = ctx.global_rank == self.leader
        n = len(requests)
        dev = eng.device
        tok_dev = torch.zeros(2, dtype=torch.int32, device=dev)
        tok_host = torch.zeros(2, dtype=torch.int32).pin_memory()
        act = torch.zeros(3, dtype=torch.int64)          # leader's action: launch ingest, join, step
        rows: list[int] = []                             # request index of each active row
        left: dict[int, int] = {}                        # tokens still to produce per request
        blocks_of: dict[int, list] = {}
        inflight: Optional[dict] = None                  # the request being ingested
        steps: deque = deque()                           # events of the steps in flight
        finishing: deque = deque()                       # (index, event, pinned tokens, n)
        nxt = 0                                          # next request to ingest
        retired = 0                                      # requests whose last step has been issued

        while retired < n:
            if lead:
                launch = join = 0
                if inflight is None and nxt < n and len(rows) < dec.rows:
                    need = eng.kv.blocks_for(int(requests[nxt].prompt.numel()) + requests[nxt].max_new)
                    if eng.kv.num_free() >= need and self.store.check([self._key("launched", nxt)]):
                        launch = 1
                if inflight is not None and inflight["ev"].query():
                    join = 1
                act[0], act[1], act[2] = launch, join, 1 if rows else 0
            if ctx.tp_size > 1:
                dist.broadcast(act, src=self.leader, group=self.dec_group)
            launch, join, step = (int(v) for v in act.tolist())
            if launch:
                i = nxt
                nxt += 1
                req = requests[i]
                prof = self._wait_key(self._key("decision", i))
                recs[i].profile = prof
                seq, slot = eng._next_seq()
                T = int(req.prompt.numel())
                blocks = eng.kv.allocate(T + req.max_new)
                table = eng.kv.block_table(blocks, eng.max_blocks)
                ist = eng.ingest_stream
                # blocks released by finished rows are not read by any queued step
                ist.wait_stream(eng.compute)
                k = i % 2
                with torch.cuda.stream(ist):
                    eng._ingest_all(T, slot, seq, prof, table, max_ctas=self.ingest_ctas)
                    eng._take_token(slot, seq, tok_dev[k:k + 1])
                    eng._return_credit(slot, seq)
                    tok_host[k:k + 1].copy_(tok_dev[k:k + 1], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(ist)
                inflight = {"i": i, "ev": ev, "k": k, "blocks": blocks, "T": T}
            if join:
                f, inflight = inflight, None
                f["ev"].synchronize()
                i = f["i"]
                t = self._now_ms() - recs[i].arrival_ms
                recs[i].kv_ready_ms = recs[i].first_token_ms = t
                if lead:
                    self.store.set(self._key("ingested", i), json.dumps({"kv_ready_ms": t}))
                row = len(rows)
                rows.append(i)
                eng.compute.wait_stream(eng.ingest_stream)
                dec.join(row, tok_dev[f["k"]:f["k"] + 1], f["T"], f["blocks"])
                left[i] = requests[i].max_new - 1
                blocks_of[i] = f["blocks"]
            if step and rows:
                dec.step(len(rows))
                e = torch.cuda.Event()
                e.record(eng.compute)
                steps.append(e)
                for i in rows:
                    left[i] -= 1
            # requests with all their tokens issued leave the batch
            for r in sorted((r for r, i in enumerate(rows) if left[i] <= 0), reverse=True):
                i = rows[r]
                nt = requests[i].max_new
                host = torch.empty(nt, dtype=torch.int32).pin_memory()
                host.copy_(dec.out[r, :nt], non_blocking=True)
                e = torch.cuda.Event()
                e.record(eng.compute)
                finishing.append((i, e, host))
                last = len(rows) - 1
                if r != last:
                    dec.move(last, r)
                    rows[r] = rows[last]
                dec.clear(last)
                rows.pop()
                eng.kv.release(blocks_of.pop(i))
                retired += 1
            while len(steps) > 2:
                steps.popleft().synchronize()
            while finishing and finishing[0][1].query():
                i, e, host = finishing.popleft()
                recs[i].done_ms = self._now_ms() - recs[i].arrival_ms
                recs[i].tokens = host.tolist()
            if not (launch or join or step):
                time.sleep(self.poll_s)
        while finishing:
            i, e, host = finishing.popleft()
            e.synchronize()
            recs[i].done_ms = self._now_ms() - recs[i].arrival_ms
            recs[i].tokens = host.tolist()


def merge_records(ctx, recs: list) -> list:
    """Combine every rank's records (max over ranks of each time; tokens
    from the decode leader).  Collective over ``ctx.cpu_group``."""
    if not ctx.distributed:
        return recs
    allr: list = [None] * ctx.world_size
    dist.all_gather_object(allr, recs, group=ctx.cpu_group)
    out = []
    for i, r in enumerate(recs):
        m = RequestRecord(r.index, r.arrival_ms, r.profile)
        for f in ("launch_ms", "prefill_ms", "kv_ready_ms", "first_token_ms", "done_ms"):
            vals = [getattr(rr[i], f) for rr in allr if getattr(rr[i], f) == getattr(rr[i], f)]
            setattr(m, f, max(vals) if vals else float("nan"))
        m.tokens = next((rr[i].tokens for rr in allr if rr[i].tokens is not None), None)
        out.append(m)
    return out


def poisson_schedule(n: int, rate_per_s: float, seed: int = 0) -> list[float]:
    """Arrival times (s) of a seeded Poisson process (all at 0 when rate <= 0)."""
    import random
    rng = random.Random(seed)
    t, out = 0.0, []
    for _ in range(n):
        t += rng.expovariate(rate_per_s) if rate_per_s > 0 else 0.0
        out.append(t)
    return out
