"""Fused random-sign Hadamard + min-max quantiser (config ``impl``
``"tilelang_fused"``, kept as the selector name for profile compatibility;
behaviour of kvserve_v1/compression/quantizer/tilelang_quantizer.py).

Keys are quantised per channel and values per token over each precision
section; the Hadamard transform is part of the operator, so pipelines that
select it drop their separate Hadamard stage (see the adapter).  On CUDA the
operator is the product sm_100a frame kernel run with 8-bit sections (one
symbol per byte); the modular pipeline's codec then packs the symbols.  The
dequantiser rebuilds a frame and runs the fused decode kernel, which writes
the output through an identity block table.  CPU tensors use the CPU oracle.

Level semantics follow the product path: ``*_max_value`` levels, symbols in
``[0, max_value - 1]``.
"""
from __future__ import annotations

from typing import Any, Optional

import numpy as np
import torch

from ..components import Quantizer
from ..heads import (get_scores, low_precision_mask, pack_sign_bits, rademacher_signs, section_orders,
                     tp_slice_mask)

_ROUTING = frozenset({"impl", "quantizer_impl", "tp_rank", "tensor_parallel_size"})


class FusedHadamardQuantizer(Quantizer):
    supports_out_buffer = True

    def __init__(self, **kwargs: Any) -> None:
        self._cfg: dict = {}
        self._validate(kwargs)
        self._cfg = dict(kwargs)
        self._state = None
        self._masks: dict = {}

    @staticmethod
    def _validate(cfg: dict) -> None:
        if cfg.get("axis_key", "channel") != "channel" or cfg.get("axis_value", "token") != "token":
            raise ValueError("the fused quantizer requires axis_key='channel' and axis_value='token'")
        if cfg.get("quant_type", "minmax") != "minmax":
            raise ValueError("the fused quantizer supports quant_type='minmax' only")
        if cfg.get("split_type", "head") not in ("head", "layer"):
            raise ValueError("split_type must be 'head' or 'layer'")

    def update_params(self, **kwargs: Any) -> None:
        kwargs = {k: v for k, v in kwargs.items() if k != "out"}
        if not kwargs:
            return
        merged = {**self._cfg, **kwargs}
        self._validate(merged)
        if merged != self._cfg:
            self._cfg = merged
            self._masks.clear()

    # ----------------------------------------------------------------- config
    @property
    def seed(self) -> int:
        s = self._cfg.get("base_seed", self._cfg.get("seed", 0x3333))
        return int(s)

    def _levels(self) -> tuple[tuple[int, int], tuple[int, int]]:
        c = self._cfg
        return ((int(c.get("low_key_max_value", 6)), int(c.get("high_key_max_value", 12))),
                (int(c.get("low_value_max_value", 4)), int(c.get("high_value_max_value", 8))))

    def _layer_order(self, layer_id: int, heads: int) -> tuple[torch.Tensor, int]:
        key = (layer_id, heads)
        hit = self._masks.get(key)
        if hit is not None:
            return hit
        c = self._cfg
        scores = get_scores(c.get("model_name"), int(c.get("num_layers", 0)), int(c.get("num_kv_heads", 0)),
                            c.get("score_path"))
        if scores.shape[0] <= layer_id:
            scores = get_scores(None, layer_id + 1, heads)
        mask = low_precision_mask(scores, float(c.get("hybrid_ratio", 0.8)), c.get("split_type", "head"))
        mask = tp_slice_mask(mask, heads, int(c.get("tp_rank", 0)), int(c.get("tensor_parallel_size", 1)))
        order, n_low = section_orders(mask[layer_id:layer_id + 1])
        hit = (order[0], int(n_low[0]))
        self._masks[key] = hit
        return hit

    def _spec(self, T: int, H: int, D: int, n_low: int):
        from ...ops.kv_codec import FrameSpec
        lv = self._levels()
        return FrameSpec(T, H, D, n_low, ((8, 8), (8, 8)), lv)

    # --------------------------------------------------------------- quantize
    def quantize(self, layer_id: int, tensor: torch.Tensor, out: Optional[torch.Tensor] = None,
                 **kwargs: Any) -> tuple[torch.Tensor, dict]:
        from ...ops import kv_codec as kc
        if kwargs:
            self.update_params(**kwargs)
        _, B, S, H, D = tensor.shape
        T = B * S
        order, n_low = self._layer_order(layer_id, H)
        spec = self._spec(T, H, D, n_low)
        lay = kc.frame_layout(spec)
        signs = rademacher_signs(self.seed, layer_id, H, D)
        k = tensor[0].reshape(T, H, D)
        v = tensor[1].reshape(T, H, D)
        if tensor.is_cuda:
            frame = torch.empty(lay.frame_bytes, dtype=torch.uint8, device=tensor.device)
            if self._state is None or self._state.device != tensor.device:
                self._state = kc.EncoderState(tensor.device)
            kc.encode_layer(k.contiguous(), v.contiguous(), spec, order.to(tensor.device),
                            pack_sign_bits(signs).to(tensor.device), frame.data_ptr(), self._state,
                            seq=1, layer=0)
        else:
            frame = torch.from_numpy(np.frombuffer(bytes(kc.cpu_encode_frame(k, v, spec, order, signs)),
                                                   dtype=np.uint8).copy())
        if out is None:
            out = torch.empty((2, B, S, H, D), dtype=torch.uint8, device=tensor.device)
        for p in range(2):
            secs = []
            for s in range(2):
                hs = spec.section_heads(s)
                if hs:
                    off = lay.payload[p][s] + 16
                    secs.append(frame[off:off + T * hs * D].view(T, hs, D))
            out[p].copy_(torch.cat(secs, dim=1).view(B, S, H, D))
        kaux = frame[lay.k_aux:lay.k_aux + 4 * H * D].view(torch.bfloat16)
        vmin, vscale = [], []
        for s in range(2):
            if spec.section_heads(s):
                a = frame[lay.v_aux[s]:lay.v_aux[s] + 4 * T].view(torch.bfloat16)
                vmin.append(a[:T].clone())
                vscale.append(a[T:].clone())
        meta = {"format": "kvs_fused_v1", "n_low": n_low, "levels": [list(x) for x in self._levels()],
                "key_min": kaux[:H * D].clone(), "key_scale": kaux[H * D:].clone(),
                "value_min": vmin, "value_scale": vscale,
                "original_dtype": str(tensor.dtype).replace("torch.", "")}
        return out, meta

    def dequantize(self, layer_id: int, tensor: torch.Tensor, meta: Any, **kwargs: Any) -> torch.Tensor:
        from ...ops import kv_codec as kc
        if meta.get("format") != "kvs_fused_v1":
            raise ValueError("not a fused-quantizer payload")
        _, B, S, H, D = tensor.shape
        T = B * S
        order, n_low = self._layer_order(layer_id, H)
        if int(meta["n_low"]) != n_low:
            raise ValueError("fused payload section split does not match this quantizer")
        spec = self._spec(T, H, D, n_low)
        lay = kc.frame_layout(spec)
        signs = rademacher_signs(self.seed, layer_id, H, D)
        frame = torch.zeros(lay.frame_bytes, dtype=torch.uint8, device=tensor.device)
        hdr = np.zeros(16, dtype=np.uint32)
        hdr[:8] = [kc.FRAME_MAGIC, 1, 0, T, H, D, n_low, 1]
        frame[:64].copy_(torch.from_numpy(hdr.view(np.uint8).copy()))
        frame[lay.k_aux:lay.k_aux + 2 * H * D].view(torch.bfloat16).copy_(meta["key_min"])
        frame[lay.k_aux + 2 * H * D:lay.k_aux + 4 * H * D].view(torch.bfloat16).copy_(meta["key_scale"])
        si = 0
        for s in range(2):
            if spec.section_heads(s):
                frame[lay.v_aux[s]:lay.v_aux[s] + 2 * T].view(torch.bfloat16).copy_(meta["value_min"][si])
                frame[lay.v_aux[s] + 2 * T:lay.v_aux[s] + 4 * T].view(torch.bfloat16).copy_(meta["value_scale"][si])
                si += 1
        for p in range(2):
            sym = tensor[p].reshape(T, H, D)
            h0 = 0
            for s in range(2):
                hs = spec.section_heads(s)
                if hs:
                    off = lay.payload[p][s]
                    frame[off:off + 16].copy_(torch.frombuffer(bytearray(kc.bitpack_header(8, T * hs * D)),
                                                               dtype=torch.uint8))
                    frame[off + 16:off + 16 + T * hs * D].view(T, hs, D).copy_(sym[:, h0:h0 + hs])
                    h0 += hs
        dtype = getattr(torch, meta.get("original_dtype", "bfloat16"))
        if tensor.is_cuda:
            out = torch.empty((1, 2, B, S, H, D), dtype=torch.bfloat16, device=tensor.device)
            status = torch.zeros(4, dtype=torch.int32, device=tensor.device)
            table = torch.arange(B, dtype=torch.int32, device=tensor.device)
            kc.decode_layers(frame.data_ptr(), lay.frame_bytes, spec, order.view(1, H).to(tensor.device),
                             pack_sign_bits(signs).view(1, H, D // 32).to(tensor.device), out, table, status,
                             seq=1)
            return out[0].to(dtype)
        kd, vd = kc.cpu_decode_frame(frame.numpy().tobytes(), spec, order, signs)
        return torch.stack([kd.view(B, S, H, D), vd.view(B, S, H, D)]).to(dtype)
