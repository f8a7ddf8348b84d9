"""Layer-streamed KV hand-off of the PD engine (the product hot path).

``TransferProfile`` is the fused-path view of a compression profile (the
same ``configs/compression`` JSON the modular pipeline uses): per-section
levels for K and V, the head split and the Hadamard seed — or ``raw`` for an
uncompressed bf16 hand-off through the same frame machinery.

``KVTransfer`` owns, for one prefill->decode channel, the per-layer head
orders / section sizes / sign bits and issues the fused kernels:

* prefill rank: ``encode(layer)`` right after layer ``l``'s K/V are written,
  on a side stream, so the push of layer ``l`` overlaps layers ``l+1..``;
* decode rank: ``ingest_all`` launches one persistent fused decode over all
  layers that waits (bounded) on each layer's publish flag; in a colocated
  deployment ``ingest_layer`` is stream-ordered right after the encode.

The reference sends every layer after the whole prefill
(kvserve_v1/connector/compressed_kv_connector.py:393-497, layer-wise
``wait_for_layer_load`` is a no-op at :374-375); streaming is this design's.
"""
from __future__ import annotations

import copy
from dataclasses import dataclass, field
from typing import Any, Optional

import torch

from ..compression.heads import (get_scores, low_precision_mask, pack_sign_bits, rademacher_signs,
                                 section_orders, tp_slice_mask)
from ..ops import kv_codec as kc

DEFAULT_SEED = 3237919422
RZE_CHUNK = 16384


@dataclass(frozen=True)
class TransferProfile:
    compressed: bool = True
    seed: int = DEFAULT_SEED
    hybrid_ratio: float = 0.8
    split_type: str = "head"
    key_levels: tuple = (6, 12)     # (low section, high section)
    value_levels: tuple = (4, 8)
    score_model: Optional[str] = None
    score_path: Optional[str] = None
    lossless: bool = False          # kvs-rze-v1 stage after the frame (the profile's lossless codec)

    @classmethod
    def raw(cls) -> "TransferProfile":
        return cls(compressed=False)

    @classmethod
    def from_compression(cls, spec: Any, model_name: Optional[str] = None) -> "TransferProfile":
        """From ``kv_connector_extra_config["compression"]``: ``None`` (raw),
        ``"default"`` or a custom pipeline dict."""
        if spec is None:
            return cls.raw()
        if spec == "default":
            from ..compression.manager import get_default_compression_config
            spec = get_default_compression_config()
        if not isinstance(spec, dict):
            raise TypeError("compression spec must be None, 'default' or a dict")
        if not spec.get("enabled", True) or "quantizer" not in spec.get("pipeline", ["quantizer"]):
            return cls.raw()
        qc = spec.get("quantizer_config") or {}
        tc = spec.get("transformer_config") or {}
        cc = spec.get("codec_config") or {}
        lossless = "codec" in spec.get("pipeline", []) and cc.get("codec_type", "bitpack") != "bitpack"
        seed = qc.get("base_seed", qc.get("seed", tc.get("seed", DEFAULT_SEED)))
        return cls(compressed=True, seed=int(seed), hybrid_ratio=float(qc.get("hybrid_ratio", 0.8)),
                   split_type=qc.get("split_type", "head"),
                   key_levels=(int(qc.get("low_key_max_value", 6)), int(qc.get("high_key_max_value", 12))),
                   value_levels=(int(qc.get("low_value_max_value", 4)), int(qc.get("high_value_max_value", 8))),
                   score_model=qc.get("model_name") or model_name, score_path=qc.get("score_path"),
                   lossless=lossless)

    def to_compression(self) -> Optional[dict]:
        if not self.compressed:
            return None
        return {"enabled": True, "pipeline": ["quantizer", "codec"],
                "quantizer_config": {"impl": "tilelang_fused", "base_seed": self.seed,
                                     "hybrid_ratio": self.hybrid_ratio, "split_type": self.split_type,
                                     "low_key_max_value": self.key_levels[0], "high_key_max_value": self.key_levels[1],
                                     "low_value_max_value": self.value_levels[0],
                                     "high_value_max_value": self.value_levels[1],
                                     "model_name": self.score_model, "axis_key": "channel", "axis_value": "token"},
                "codec_config": {"codec_type": "lc", "lc_algorithm": "kvs-rze-v1"} if self.lossless else
                {"codec_type": "bitpack", "bitpack_bits": 8}}


class KVTransfer:
    def __init__(self, profile: TransferProfile, num_layers: int, num_kv_heads_total: int, local_heads: int,
                 head_dim: int, tp_rank: int, tp_size: int, device, max_tokens: int,
                 score_model_name: Optional[str] = None):
        self.profile = profile
        self.L, self.H, self.D = num_layers, local_heads, head_dim
        self.device = torch.device(device)
        if profile.compressed:
            scores = get_scores(profile.score_model or score_model_name, num_layers, num_kv_heads_total,
                                profile.score_path)
            if scores.shape != (num_layers, num_kv_heads_total):
                scores = get_scores(None, num_layers, num_kv_heads_total)
            mask = low_precision_mask(scores, profile.hybrid_ratio, profile.split_type)
            mask = tp_slice_mask(mask, local_heads, tp_rank, tp_size)
        else:
            mask = torch.zeros((num_layers, local_heads), dtype=torch.bool)
        orders, n_lows = section_orders(mask)
        self.orders_cpu, self.n_lows_cpu = orders, n_lows
        self.orders = orders.to(self.device)
        self.n_lows = n_lows.to(self.device)
        signs = torch.stack([rademacher_signs(profile.seed, l, local_heads, head_dim) for l in range(num_layers)])
        self.sign_bits = pack_sign_bits(signs).to(self.device)   # [L, H, D/32]
        self.max_tokens = max_tokens
        # bytes of the largest frame, and the bytes a slot reserves per layer
        # (the lossless codec's worst case when the profile has that stage)
        self.frame_bytes_max = max(kc.frame_layout(self.spec(l, max_tokens)).frame_bytes for l in range(num_layers))
        self.frame_stride = self.frame_bytes_max
        self._state: Optional[kc.EncoderState] = None
        if profile.lossless:
            from ..ops import ext
            cap = ext().rze_max_encoded_bytes(self.frame_bytes_max, RZE_CHUNK)
            self.frame_stride = (cap + 255) // 256 * 256
            dev = self.device
            self._stage = torch.empty(self.frame_bytes_max, dtype=torch.uint8, device=dev)
            self._scratch = torch.empty(ext().rze_scratch_bytes(self.frame_bytes_max, RZE_CHUNK), dtype=torch.uint8,
                                        device=dev)
            self._total = torch.zeros(1, dtype=torch.int64, device=dev)
            self.wire_bytes = torch.zeros(1, dtype=torch.int64, device=dev)   # encoded bytes of the last request

    def spec(self, layer: int, T: int) -> kc.FrameSpec:
        n_low = int(self.n_lows_cpu[layer])
        p = self.profile
        return kc.spec_from_profile(T, self.H, self.D, n_low, p.key_levels, p.value_levels, raw=not p.compressed)

    def max_spec(self, T: int) -> kc.FrameSpec:
        """The spec of the largest frame (used as the decode kernel's base geometry)."""
        best = max(range(self.L), key=lambda l: kc.frame_layout(self.spec(l, T)).frame_bytes)
        return self.spec(best, T)

    def payload_bytes(self, T: int) -> int:
        return sum(kc.frame_layout(self.spec(l, T)).frame_bytes for l in range(self.L))

    def raw_bytes(self, T: int) -> int:
        return 2 * self.L * T * self.H * self.D * 2

    # ------------------------------------------------------------ prefill
    def encode(self, layer: int, k: torch.Tensor, v: torch.Tensor, frame_ptr: int, flag_ptr: int, seq: int,
               pacing: Optional[torch.Tensor] = None, rate_bytes_per_ns: float = 0.0, max_ctas: int = 222,
               trace: Optional[torch.Tensor] = None) -> None:
        if self._state is None:
            self._state = kc.EncoderState(self.device, max_tokens=self.max_tokens)
        if self.D == 128 and getattr(self, "_hs_table", None) is None:
            # signed transform table of every (layer, head) for the tensor-core encoder
            from ..ops import ext
            self._hs_table = ext().kv_signed_hadamard(self.sign_bits.reshape(-1, 4).contiguous())
        spec = self.spec(layer, k.shape[0])
        lossless = self.profile.lossless
        # with the lossless stage the frame goes to local staging first and
        # the codec's output is what lands in the slot, published afterwards
        kc.encode_layer(k, v, spec, self.orders[layer], self.sign_bits[layer],
                        self._stage.data_ptr() if lossless else frame_ptr, self._state,
                        flag_ptr=0 if lossless else flag_ptr, seq=seq, layer=layer, pacing=pacing,
                        rate_bytes_per_ns=rate_bytes_per_ns, max_ctas=max_ctas,
                        hs_table=getattr(self, "_hs_table", None), hs_row0=layer * self.H,
                        trace_ptr=trace[layer].data_ptr() if trace is not None else 0)
        if lossless:
            from .. import ops
            n = kc.frame_layout(spec).frame_bytes
            out = ops.ext().tensor_from_ptr(int(frame_ptr), [self.frame_stride], ops.dtype_code(torch.uint8),
                                            self.device.index)
            ops.count_launches(3)
            ops.ext().rze_encode(self._stage[:n], out, self._scratch, self._total, RZE_CHUNK)
            if layer == 0:
                self.wire_bytes.zero_()
            self.wire_bytes.add_(self._total)
            if flag_ptr:
                ops.count_launches(1)
                ops.ext().store_release_u32(int(flag_ptr), int(seq))

    def _unpack_lossless(self, layer: int, T: int, frame_ptr: int, flag_ptr: int, seq: int, timeout_ns: int,
                         status: torch.Tensor) -> int:
        """Lossless stage of the decode side: (wait for the layer's flag, then)
        decode the slot's codec payload into local staging; returns the
        staging address of the frame."""
        from .. import ops
        if flag_ptr:
            ops.count_launches(1)
            ops.ext().wait_flag(int(flag_ptr), int(seq), int(timeout_ns), status)
        n = kc.frame_layout(self.spec(layer, T)).frame_bytes
        src = ops.ext().tensor_from_ptr(int(frame_ptr), [self.frame_stride], ops.dtype_code(torch.uint8),
                                        self.device.index)
        ops.count_launches(2)
        ops.ext().rze_decode(src, self._stage[:n], self._scratch, RZE_CHUNK)
        return self._stage.data_ptr()

    # ------------------------------------------------------------- decode
    def ingest_layer(self, layer: int, T: int, frame_ptr: int, kv_cache: torch.Tensor, block_table: torch.Tensor,
                     status: torch.Tensor, seq: int, tok_offset: int = 0, trace: Optional[torch.Tensor] = None) -> None:
        spec = self.spec(layer, T)
        if self.profile.lossless:
            frame_ptr = self._unpack_lossless(layer, T, frame_ptr, 0, seq, 0, status)
        kc.decode_layers(frame_ptr, kc.frame_layout(spec).frame_bytes, spec, self.orders, self.sign_bits, kv_cache,
                         block_table, status, tok_offset=tok_offset, seq=seq, layer_begin=layer, num_layers=1,
                         trace_ptr=trace.data_ptr() if trace is not None else 0)

    def ingest_all(self, T: int, slot_base: int, frame_stride: int, flags_ptr: int, kv_cache: torch.Tensor,
                   block_table: torch.Tensor, status: torch.Tensor, seq: int, timeout_ns: int,
                   tok_offset: int = 0, max_ctas: int = 148, trace: Optional[torch.Tensor] = None) -> None:
        if self.profile.lossless:
            # per layer: bounded flag wait, codec decode into staging, frame decode
            for l in range(self.L):
                ptr = self._unpack_lossless(l, T, slot_base + l * frame_stride, flags_ptr + 4 * l, seq, timeout_ns,
                                            status)
                spec = self.spec(l, T)
                kc.decode_layers(ptr, kc.frame_layout(spec).frame_bytes, spec, self.orders, self.sign_bits, kv_cache,
                                 block_table, status, tok_offset=tok_offset, seq=seq, layer_begin=l, num_layers=1,
                                 max_ctas=max_ctas, trace_ptr=trace.data_ptr() if trace is not None else 0)
            return
        kc.decode_layers(slot_base, frame_stride, self.max_spec(T), self.orders, self.sign_bits, kv_cache,
                         block_table, status, tok_offset=tok_offset, flags_ptr=flags_ptr, seq=seq, layer_begin=0,
                         num_layers=self.L, timeout_ns=timeout_ns, max_ctas=max_ctas, n_lows=self.n_lows,
                         trace_ptr=trace.data_ptr() if trace is not None else 0)
