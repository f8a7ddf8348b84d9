"""Llama / Qwen2-style decoder running entirely on the kvserve_b200 sm_100a
kernels (tcgen05 GEMM, tcgen05 flash attention, paged decode attention,
fused RoPE + KV write, RMSNorm, SiLU-mul, weight-streaming GEMV).

Tensor parallel (Megatron layout): QKV and gate/up are column-parallel, O and
down row-parallel followed by an NCCL all-reduce over NVLink; the LM head is
vocab-parallel with a distributed greedy argmax.  KV heads are replicated when
``tp_size > num_kv_heads``.  Weights are random-initialised per shard from a
deterministic seed, so the prefill and decode ranks of one TP index hold
identical shards without any checkpoint; ``save`` / ``load`` write and read
one safetensors file per shard for runs that want the weights on disk.
"""
from __future__ import annotations

import hashlib
import math
import os
from dataclasses import dataclass, fields
from typing import Callable, Optional

import torch
import torch.distributed as dist

from .. import ops
from ..utils.trace import nvtx_pop, nvtx_push
from .config import ModelConfig


def _seed(*parts) -> int:
    h = hashlib.sha256("|".join(str(p) for p in parts).encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


def rope_cache(max_pos: int, head_dim: int, theta: float, device) -> torch.Tensor:
    """[max_pos, head_dim] fp32: cos of the D/2 frequencies, then their sin."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.cat([f.cos(), f.sin()], dim=-1).float().to(device)


@dataclass
class LayerWeights:
    qkv: torch.Tensor
    qkv_bias: Optional[torch.Tensor]
    o: torch.Tensor
    gate_up: torch.Tensor
    down: torch.Tensor
    in_norm: torch.Tensor
    post_norm: torch.Tensor


class LlamaShard:
    def __init__(self, cfg: ModelConfig, tp_rank: int = 0, tp_size: int = 1, device=None, seed: int = 0,
                 tp_group=None, max_position: int = 32768, init_std: float = 0.02):
        self.cfg = cfg
        self.tp_rank, self.tp_size, self.tp_group = tp_rank, tp_size, tp_group
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if cfg.num_q_heads % tp_size or cfg.intermediate % tp_size or cfg.vocab % tp_size:
            raise ValueError("model dims must divide the TP size")
        self.hq = cfg.num_q_heads // tp_size
        if tp_size <= cfg.num_kv_heads:
            if cfg.num_kv_heads % tp_size:
                raise ValueError("kv heads must divide the TP size")
            self.hkv = cfg.num_kv_heads // tp_size
            self.kv_head_offset = tp_rank * self.hkv
        else:  # replicated KV heads
            self.hkv = 1
            self.kv_head_offset = tp_rank * cfg.num_kv_heads // tp_size
        self.inter = cfg.intermediate // tp_size
        self.gu_block = ops.GATE_UP_BLOCK if self.inter % ops.GATE_UP_BLOCK == 0 else 0
        self.vocab_local = cfg.vocab // tp_size
        self.vocab_begin = tp_rank * self.vocab_local
        self.D = cfg.head_dim
        self.scale = 1.0 / math.sqrt(self.D)
        self.seed = seed
        self.init_std = init_std
        dev = self.device
        self.layers: list[LayerWeights] = []
        for l in range(cfg.num_layers):
            qkv_rows = (self.hq + 2 * self.hkv) * self.D
            self.layers.append(LayerWeights(
                qkv=self._rand((qkv_rows, cfg.hidden), l, "qkv"),
                qkv_bias=self._rand((qkv_rows,), l, "qkv_bias") if cfg.qkv_bias else None,
                o=self._rand((cfg.hidden, self.hq * self.D), l, "o"),
                # [2I, K], gate/up rows interleaved in blocks of ops.GATE_UP_BLOCK
                # (the fused SiLU GEMM layout) when I allows it
                gate_up=self._rand((2 * self.inter, cfg.hidden), l, "gate_up"),
                down=self._rand((cfg.hidden, self.inter), l, "down"),
                in_norm=torch.ones(cfg.hidden, dtype=torch.bfloat16, device=dev),
                post_norm=torch.ones(cfg.hidden, dtype=torch.bfloat16, device=dev),
            ))
        self.embed = self._rand((cfg.vocab, cfg.hidden), -1, "embed", tp_shared=True, std=1.0)
        self.lm_head = self._rand((self.vocab_local, cfg.hidden), -1, "lm_head")
        self.final_norm = torch.ones(cfg.hidden, dtype=torch.bfloat16, device=dev)
        self.cos_sin = rope_cache(max_position, self.D, cfg.rope_theta, dev)
        # fused GEMM + all-reduce workspace (parallel.tp_allreduce) and the
        # decode-step collective workspace (parallel.decode_allreduce), both
        # attached by the engine
        self.tp_ar = None
        self.decode_coll = None

    # ------------------------------------------------------------------ init
    def _rand(self, shape, layer, name, tp_shared=False, std=None) -> torch.Tensor:
        g = torch.Generator(device=self.device)
        g.manual_seed(_seed(self.cfg.name, self.seed, layer, name, 0 if tp_shared else self.tp_rank,
                            1 if tp_shared else self.tp_size))
        t = torch.empty(shape, dtype=torch.bfloat16, device=self.device)
        t.normal_(0.0, self.init_std if std is None else std, generator=g)
        return t

    # ----------------------------------------------------------- checkpoint
    CHECKPOINT_FORMAT = "kvserve_b200-llama-shard-v1"

    def state_dict(self) -> dict:
        """This shard's weights by name (views, not copies): ``embed``,
        ``lm_head``, ``final_norm`` and ``layers.<l>.<field>`` in the layout
        the kernels read (gate/up rows interleaved in GATE_UP_BLOCK blocks)."""
        sd = {"embed": self.embed, "lm_head": self.lm_head, "final_norm": self.final_norm}
        for l, lw in enumerate(self.layers):
            for f in fields(LayerWeights):
                t = getattr(lw, f.name)
                if t is not None:
                    sd[f"layers.{l}.{f.name}"] = t
        return sd

    def load_state_dict(self, sd: dict) -> None:
        """Copy ``sd`` into the shard's tensors in place, so CUDA graphs and
        the collective workspaces that hold their addresses stay valid; the
        names, shapes and dtypes must match exactly."""
        own = self.state_dict()
        missing, unexpected = sorted(own.keys() - sd.keys()), sorted(sd.keys() - own.keys())
        if missing or unexpected:
            raise KeyError(f"checkpoint does not match the shard: missing {missing[:4]}, unexpected {unexpected[:4]}")
        for name, t in own.items():
            src = sd[name]
            if tuple(src.shape) != tuple(t.shape) or src.dtype != t.dtype:
                raise ValueError(f"{name}: checkpoint {tuple(src.shape)} {src.dtype}, shard {tuple(t.shape)} {t.dtype}")
            t.copy_(src)

    @staticmethod
    def shard_path(prefix: str, tp_rank: int, tp_size: int) -> str:
        return f"{prefix}.tp{tp_rank}of{tp_size}.safetensors"

    def save(self, prefix: str) -> str:
        """Write this shard to ``<prefix>.tp<rank>of<size>.safetensors``
        (atomically: ranks of two engines that hold the same shard may write
        it at once) and return the path."""
        from safetensors.torch import save_file
        path = self.shard_path(prefix, self.tp_rank, self.tp_size)
        tmp = f"{path}.{os.getpid()}.tmp"
        meta = {"format": self.CHECKPOINT_FORMAT, "model": self.cfg.name, "seed": str(self.seed),
                "tp_rank": str(self.tp_rank), "tp_size": str(self.tp_size)}
        save_file({k: v.contiguous() for k, v in self.state_dict().items()}, tmp, metadata=meta)
        os.replace(tmp, path)
        return path

    def load(self, prefix: str) -> None:
        """Load the shard this rank holds from ``save``'s file of the same TP
        geometry."""
        from safetensors import safe_open
        path = self.shard_path(prefix, self.tp_rank, self.tp_size)
        with safe_open(path, framework="pt", device=str(self.device)) as f:
            meta = f.metadata() or {}
            if meta.get("format") != self.CHECKPOINT_FORMAT or meta.get("model") != self.cfg.name:
                raise ValueError(f"{path} holds {meta.get('model')!r} in format {meta.get('format')!r}, "
                                 f"not {self.cfg.name!r}")
            self.load_state_dict({k: f.get_tensor(k) for k in f.keys()})

    def weight_bytes(self) -> int:
        n = sum(t.numel() for lw in self.layers for t in (lw.qkv, lw.o, lw.gate_up, lw.down))
        return 2 * (n + self.embed.numel() + self.lm_head.numel())

    # ------------------------------------------------------------- helpers
    def _all_reduce(self, x: torch.Tensor) -> None:
        if self.tp_size > 1:
            dist.all_reduce(x, group=self.tp_group)

    def _row_parallel(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """``x @ w.T`` summed over the TP group: one fused GEMM + peer-memory
        all-reduce launch where the workspace takes the shape, else the GEMM
        followed by an NCCL all-reduce."""
        ar = self.tp_ar
        if ar is not None and ar.accepts(x.shape[0], w.shape[0]):
            return ar.gemm_allreduce(x, w)
        y = ops.linear(x, w)
        self._all_reduce(y)
        return y

    def _qkv(self, h: torch.Tensor, lw: LayerWeights) -> torch.Tensor:
        return ops.linear(h, lw.qkv, bias=lw.qkv_bias)

    def _mlp(self, h: torch.Tensor, lw: LayerWeights, site: Optional[int] = None) -> torch.Tensor:
        if self.gu_block and h.shape[0] > ops.GEMV_MAX_M:
            a = ops.gemm_silu(h, lw.gate_up)
        else:
            a = ops.silu_mul(ops.linear(h, lw.gate_up), block=self.gu_block)
        return self._decode_row_parallel(a, lw.down, site)

    def decode_sites(self) -> int:
        """Launch sites of the fused decode collectives in one step: the two
        row-parallel projections of every layer and the LM head."""
        return 2 * self.cfg.num_layers + 1

    def _decode_row_parallel(self, x: torch.Tensor, w: torch.Tensor, site: Optional[int]) -> torch.Tensor:
        dc = self.decode_coll
        if site is not None and dc is not None and dc.world > 1 and x.reshape(-1, x.shape[-1]).shape[0] <= 8:
            return dc.gemv_allreduce(x, w, site)
        return self._row_parallel(x, w)

    def greedy(self, h_last: torch.Tensor) -> torch.Tensor:
        """Greedy next token over the vocab-parallel LM head (int32 [B])."""
        logits = ops.linear(h_last, self.lm_head)
        if self.tp_size == 1:
            return ops.argmax(logits)
        vals = torch.empty(h_last.shape[0], dtype=torch.float32, device=self.device)
        idx = ops.argmax(logits, index_offset=self.vocab_begin, out_val=vals)
        both = torch.stack([vals, idx.to(torch.float32)], 0)
        gathered = torch.empty((self.tp_size,) + tuple(both.shape), dtype=both.dtype, device=self.device)
        dist.all_gather_into_tensor(gathered, both, group=self.tp_group)
        best = gathered[:, 0].argmax(0)
        return gathered[:, 1].gather(0, best[None])[0].to(torch.int32)

    # -------------------------------------------------------------- prefill
    def prefill(self, ids: torch.Tensor, positions: torch.Tensor, k_buf: torch.Tensor, v_buf: torch.Tensor,
                layer_hook: Optional[Callable[[int], None]] = None, sample: bool = False) -> Optional[torch.Tensor]:
        """Forward over a prompt chunk ``ids`` (int32 [T]) writing the rotated
        K and V of layer ``l`` into ``k_buf[l]`` / ``v_buf[l]`` (``[L, T, Hkv, D]``)
        and calling ``layer_hook(l)`` right after they are written."""
        cfg = self.cfg
        T = ids.numel()
        residual = ops.embedding(ids, self.embed)
        h = ops.rmsnorm(residual, self.layers[0].in_norm, cfg.rms_eps)
        fused_qkv = self.D == 128 and T > ops.GEMV_MAX_M
        for l, lw in enumerate(self.layers):
            nvtx_push(f"prefill L{l}")
            if fused_qkv:  # projection + bias + rotary + K/V copy in one GEMM
                qkv = ops.gemm_qkv_rope(h, lw.qkv, self.hq, self.hkv, positions, self.cos_sin, bias=lw.qkv_bias,
                                        k_dst=k_buf[l, :T], v_dst=v_buf[l, :T])
            else:
                qkv = self._qkv(h, lw)
                ops.rope_qkv(qkv, self.hq, self.hkv, self.D, positions, self.cos_sin, k_buf[l, :T],
                             v_buf[l, :T])
            if layer_hook is not None:
                layer_hook(l)
            attn = ops.flash_prefill(qkv, self.hq, self.hkv, self.scale)
            o = self._row_parallel(attn, lw.o)
            h = ops.rmsnorm(o, lw.post_norm, cfg.rms_eps, residual=residual)
            d = self._mlp(h, lw)
            nxt = self.layers[l + 1].in_norm if l + 1 < len(self.layers) else self.final_norm
            h = ops.rmsnorm(d, nxt, cfg.rms_eps, residual=residual)
            nvtx_pop()
        if not sample:
            return None
        return self.greedy(h[T - 1:T].contiguous())

    # --------------------------------------------------------------- decode
    def decode_step(self, ids: torch.Tensor, positions: torch.Tensor, slot_mapping: torch.Tensor,
                    kv_cache: torch.Tensor, block_tables: torch.Tensor, ctx_lens: torch.Tensor,
                    max_ctx: int, attn_scratch=None) -> torch.Tensor:
        """One token per sequence against the paged cache
        ``kv_cache`` ``[L, 2, num_blocks, block_size, Hkv, D]``; returns int32 [B]."""
        cfg = self.cfg
        B = ids.numel()
        nb, bs = kv_cache.shape[2], kv_cache.shape[3]
        residual = ops.embedding(ids, self.embed)
        h = ops.rmsnorm(residual, self.layers[0].in_norm, cfg.rms_eps)
        for l, lw in enumerate(self.layers):
            qkv = self._qkv(h, lw)
            kc = kv_cache[l, 0].view(nb * bs, self.hkv, self.D)
            vc = kv_cache[l, 1].view(nb * bs, self.hkv, self.D)
            ops.rope_qkv(qkv, self.hq, self.hkv, self.D, positions, self.cos_sin, kc, vc, slot_mapping=slot_mapping)
            q = qkv[:, : self.hq * self.D].view(B, self.hq, self.D)
            attn = ops.paged_decode_attention(q, kv_cache[l, 0], kv_cache[l, 1], block_tables, ctx_lens, max_ctx,
                                              self.scale, scratch=attn_scratch)
            o = self._decode_row_parallel(attn.view(B, self.hq * self.D), lw.o, 2 * l)
            h = ops.rmsnorm(o, lw.post_norm, cfg.rms_eps, residual=residual)
            d = self._mlp(h, lw, 2 * l + 1)
            nxt = self.layers[l + 1].in_norm if l + 1 < len(self.layers) else self.final_norm
            h = ops.rmsnorm(d, nxt, cfg.rms_eps, residual=residual)
        dc = self.decode_coll
        if dc is None or B > 8:
            return self.greedy(h)
        tok = dc.greedy(h, self.lm_head, self.vocab_begin, 2 * cfg.num_layers)
        dc.bump()
        return tok
