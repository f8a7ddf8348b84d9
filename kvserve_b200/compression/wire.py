"""GPU-resident wire format of modular-pipeline payloads.

The rules are those of the reference (kvserve_v1/compression/wire.py:16-289)
so that producers and consumers of either implementation agree on the
message structure:

* ``meta`` is msgpack-able: every tensor inside ``quantization_params`` is
  replaced by the placeholder ``["__kvserve_aux_tensor__", index]``;
* two or more aux tensors are coalesced into one uint8 tensor, each entry
  aligned to its itemsize, described by ``meta["aux_layout"] = {"mode":
  "coalesced_bytes", "tensors": [{storage, offset, nbytes, shape, dtype}]}``;
* a body larger than ``max_chunk_bytes`` is split into ``byte_chunks``;
  chunked manager payloads travel as ``manager_chunks``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from .manager import CompressedKVData

AUX_PLACEHOLDER = "__kvserve_aux_tensor__"


@dataclass
class CompressedWire:
    meta: dict
    body_chunks: list
    aux_tensors: list

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.body_chunks + self.aux_tensors)


def _dtype_name(t: torch.Tensor) -> str:
    return str(t.dtype).replace("torch.", "")


def _spec(t: torch.Tensor) -> dict:
    return {"shape": list(t.shape), "dtype": _dtype_name(t)}


def _pack(obj: Any, aux: list) -> Any:
    if isinstance(obj, torch.Tensor):
        aux.append(obj.contiguous())
        return [AUX_PLACEHOLDER, len(aux) - 1]
    if isinstance(obj, dict):
        return {k: _pack(v, aux) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return [_pack(v, aux) for v in obj]
    return obj


def _is_placeholder(obj: Any) -> bool:
    return isinstance(obj, list) and len(obj) == 2 and isinstance(obj[0], str) and obj[0] == AUX_PLACEHOLDER


def _unpack(obj: Any, aux: list) -> Any:
    if _is_placeholder(obj):
        return aux[int(obj[1])]
    if isinstance(obj, dict):
        return {k: _unpack(v, aux) for k, v in obj.items()}
    if isinstance(obj, list):
        return [_unpack(v, aux) for v in obj]
    return obj


def _pack_meta(meta: Any, aux: list) -> Any:
    if not isinstance(meta, dict):
        return meta
    out = dict(meta)
    if "quantization_params" in out:
        out["quantization_params"] = _pack(out["quantization_params"], aux)
    return out


def _unpack_meta(meta: Any, aux: list) -> Any:
    if isinstance(meta, dict) and "quantization_params" in meta:
        meta = dict(meta)
        meta["quantization_params"] = _unpack(meta["quantization_params"], aux)
    return meta


def coalesce_aux(meta: dict, aux: list) -> list:
    if len(aux) <= 1:
        return aux
    pieces, layout, off = [], [], 0
    dev = aux[0].device
    for t in aux:
        t = t.contiguous()
        pad = (-off) % t.element_size()
        if pad:
            pieces.append(torch.zeros(pad, dtype=torch.uint8, device=dev))
            off += pad
        b = t.reshape(-1).view(torch.uint8)
        layout.append({"storage": 0, "offset": off, "nbytes": b.numel(), "shape": list(t.shape),
                       "dtype": _dtype_name(t)})
        pieces.append(b.to(dev))
        off += b.numel()
    meta["aux_layout"] = {"mode": "coalesced_bytes", "tensors": layout}
    return [torch.cat(pieces).contiguous()]


def expand_aux(wire_aux: list, layout: Any) -> list:
    if not layout:
        return wire_aux
    if layout.get("mode") != "coalesced_bytes":
        raise ValueError(f"Unknown aux_layout mode: {layout.get('mode')}")
    if not wire_aux:
        return []
    store = wire_aux[0].contiguous().view(torch.uint8).flatten()
    out = []
    for spec in layout.get("tensors", []):
        if int(spec.get("storage", 0)) != 0:
            raise ValueError("Only single-storage aux_layout is supported")
        s, n = int(spec["offset"]), int(spec["nbytes"])
        out.append(store[s:s + n].view(getattr(torch, spec["dtype"])).reshape(spec["shape"]))
    return out


def _split_bytes(t: torch.Tensor, max_chunk: int) -> list:
    if max_chunk <= 0:
        raise ValueError("max_chunk_bytes must be positive")
    b = t.contiguous().view(torch.uint8).flatten()
    return [b[i:i + max_chunk].contiguous() for i in range(0, b.numel(), max_chunk)]


def assert_no_tensor(obj: Any) -> None:
    if isinstance(obj, torch.Tensor):
        raise TypeError("CompressedWire metadata still contains a tensor")
    if isinstance(obj, dict):
        for v in obj.values():
            assert_no_tensor(v)
    elif isinstance(obj, (list, tuple)):
        for v in obj:
            assert_no_tensor(v)


def build_wire(c: CompressedKVData, max_chunk_bytes: int) -> CompressedWire:
    aux: list = []
    if c.is_chunked:
        if not c.chunks or not c.chunk_metadata:
            raise ValueError("Chunked CompressedKVData is missing chunks or metadata")
        meta = {"is_chunked": True, "layer_id": c.layer_id, "original_size": c.original_size,
                "compressed_size": c.compressed_size, "metadata": _pack_meta(c.metadata, aux),
                "chunk_metadata": [_pack_meta(m, aux) for m in c.chunk_metadata], "body_mode": "manager_chunks"}
        body = [x.contiguous() for x in c.chunks]
    else:
        if c.compressed_tensor is None:
            raise ValueError("Non-chunked CompressedKVData is missing compressed_tensor")
        t = c.compressed_tensor.contiguous()
        nbytes = t.numel() * t.element_size()
        if nbytes > max_chunk_bytes:
            body, mode = _split_bytes(t, max_chunk_bytes), "byte_chunks"
        else:
            body, mode = [t], "single"
        meta = {"is_chunked": False, "layer_id": c.layer_id, "original_size": c.original_size,
                "compressed_size": c.compressed_size, "metadata": _pack_meta(c.metadata, aux),
                "body_mode": mode, "body_spec": _spec(t)}
    wire_aux = coalesce_aux(meta, aux)
    assert_no_tensor(meta)
    return CompressedWire(meta, body, wire_aux)


def restore_from_wire(w: CompressedWire) -> CompressedKVData:
    meta = w.meta
    aux = expand_aux(w.aux_tensors, meta.get("aux_layout"))
    inner = _unpack_meta(meta.get("metadata"), aux)
    rid = str(inner.get("request_id", "unknown")) if isinstance(inner, dict) else "unknown"
    if meta["is_chunked"]:
        return CompressedKVData(rid, int(meta.get("layer_id", -1)), None, inner, int(meta.get("original_size", 0)),
                                int(meta.get("compressed_size", 0)), True, list(w.body_chunks),
                                [_unpack_meta(m, aux) for m in meta.get("chunk_metadata", [])])
    if meta.get("body_mode") == "byte_chunks":
        b = torch.cat([x.contiguous().view(torch.uint8) for x in w.body_chunks])
        spec = meta["body_spec"]
        body = b.view(getattr(torch, spec["dtype"])).reshape(spec["shape"])
    else:
        body = w.body_chunks[0]
    return CompressedKVData(rid, int(meta.get("layer_id", -1)), body, inner, int(meta.get("original_size", 0)),
                            int(meta.get("compressed_size", 0)), False)
