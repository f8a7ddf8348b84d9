"""Fused KV-frame codec: layout, CPU oracle and the sm_100a kernel front-end.

A *frame* is one layer's K and V for one request shard (``T`` tokens, ``H``
local KV heads, head_dim ``D``), compressed with a random-sign Hadamard
transform and min-max quantisation (K per channel, V per token and section),
bit-packed into BitPack-format sections.  The byte layout is described in
``csrc/kv_frame.h``; :func:`frame_layout` computes the identical offsets in
Python so CPU code (tests, the gloo transport) can read and write frames.

Reference behaviour (re-designed): the fused K/V encode/restore of
kvserve_v1/compression/runtime/csrc/fused/kvs_fused.cu:126-388 and the hybrid
min-max quantiser kvserve_v1/compression/quantizer/kvserve_quantizer.py:171-294.
"""
from __future__ import annotations

import os

import math
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np
import torch

RAW_BITS = 16
FRAME_ALIGN = 256
HEADER_BYTES = 64
FRAME_MAGIC = 0x4653564B
BITPACK_MAGIC = 0x0150424B


def _align(x: int, a: int = FRAME_ALIGN) -> int:
    return (x + a - 1) // a * a


def bits_for_levels(levels: int) -> int:
    """Smallest bit width holding symbols ``0 .. levels-1``."""
    if levels < 2 or levels > 256:
        raise ValueError("levels must be in [2, 256]")
    return max(1, math.ceil(math.log2(levels)))


@dataclass(frozen=True)
class FrameSpec:
    """Geometry + precision of one layer frame.  ``bits[p][s]`` / ``levels[p][s]``
    for part p (0 = K, 1 = V) and section s (0 = low heads, 1 = high heads);
    ``bits == 16`` marks an uncompressed (raw bf16) section."""

    T: int
    H: int
    D: int
    n_low: int
    bits: tuple = ((4, 4), (4, 4))
    levels: tuple = ((16, 16), (16, 16))
    transform: bool = True

    def params(self) -> list[int]:
        return [self.T, self.H, self.D, self.n_low,
                self.bits[0][0], self.bits[0][1], self.bits[1][0], self.bits[1][1],
                self.levels[0][0], self.levels[0][1], self.levels[1][0], self.levels[1][1], int(self.transform)]

    def section_heads(self, s: int) -> int:
        return self.n_low if s == 0 else self.H - self.n_low

    def with_tokens(self, T: int) -> "FrameSpec":
        return FrameSpec(T, self.H, self.D, self.n_low, self.bits, self.levels, self.transform)


@dataclass(frozen=True)
class FrameLayout:
    frame_bytes: int
    k_aux: int
    v_aux: tuple
    payload: tuple  # [p][s]


def frame_layout(spec: FrameSpec) -> FrameLayout:
    """Byte offsets of every region of a frame (mirror of frame_geom_finalize)."""
    off = _align(HEADER_BYTES)
    k_quant = any(spec.section_heads(s) > 0 and spec.bits[0][s] != RAW_BITS for s in range(2))
    k_aux = off
    if k_quant:
        off = _align(off + 2 * 2 * spec.H * spec.D)
    v_aux = []
    for s in range(2):
        v_aux.append(off)
        if spec.section_heads(s) > 0 and spec.bits[1][s] != RAW_BITS:
            off = _align(off + 2 * 2 * spec.T)
    payload = [[0, 0], [0, 0]]
    for p in range(2):
        for s in range(2):
            payload[p][s] = off
            hs = spec.section_heads(s)
            if hs == 0:
                continue
            count = spec.T * hs * spec.D
            b = spec.bits[p][s]
            nbytes = count * 2 if b == RAW_BITS else (count * b + 7) // 8
            hdr = 0 if b == RAW_BITS else 16
            off = _align(off + hdr + nbytes)
    return FrameLayout(off, k_aux, tuple(v_aux), (tuple(payload[0]), tuple(payload[1])))


def spec_from_profile(T: int, H: int, D: int, n_low: int, key_levels: Sequence[int],
                      value_levels: Sequence[int], raw: bool = False) -> FrameSpec:
    """Frame spec from (low, high) level counts of keys and values.

    Profiles written for the reference give ``*_max_value``; the reference
    quantiser maps values into ``[0, max_value-1]`` (scale = range /
    (max_value - 1)), so ``levels = max_value`` and ``bits = ceil(log2(levels))``.
    """
    if raw:
        return FrameSpec(T, H, D, n_low, ((RAW_BITS, RAW_BITS), (RAW_BITS, RAW_BITS)), ((2, 2), (2, 2)))
    kl = tuple(int(x) for x in key_levels)
    vl = tuple(int(x) for x in value_levels)
    bits = ((bits_for_levels(kl[0]), bits_for_levels(kl[1])), (bits_for_levels(vl[0]), bits_for_levels(vl[1])))
    return FrameSpec(T, H, D, n_low, bits, (kl, vl))


# ----------------------------------------------------------------------------
# CPU oracle (fp32 math identical in structure to the CUDA kernels)
# ----------------------------------------------------------------------------

def hadamard_matrix(n: int) -> torch.Tensor:
    """Sylvester-ordered ±1 Hadamard matrix (H[i, j] = (-1)^popcount(i & j))."""
    i = torch.arange(n)
    bits = (i[:, None] & i[None, :])
    pc = torch.zeros_like(bits)
    b = bits.clone()
    while bool((b > 0).any()):
        pc += b & 1
        b >>= 1
    return (1 - 2 * (pc & 1)).to(torch.float32)


def _bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def _pack_bits(sym: np.ndarray, bits: int) -> bytes:
    """LSB-first packing of uint8 symbols (BitPack stream, no header): bit
    ``b`` of symbol ``i`` is bit ``i * bits + b`` of the stream, and stream
    bit ``j`` is bit ``j % 8`` of byte ``j // 8``."""
    sym = np.ascontiguousarray(sym, dtype=np.uint8).reshape(-1)
    if bits in (1, 2, 4, 8):              # whole symbols per byte: shift and add
        per = 8 // bits
        pad = (-sym.size) % per
        grp = np.concatenate([sym, np.zeros(pad, dtype=np.uint8)]).reshape(-1, per)
        shifts = (np.arange(per, dtype=np.uint8) * bits)
        return np.bitwise_or.reduce(grp << shifts, axis=1).astype(np.uint8).tobytes()
    planes = np.unpackbits(sym.reshape(-1, 1), axis=1, bitorder="little")[:, :bits]   # [n, bits]
    return np.packbits(planes.reshape(-1), bitorder="little").tobytes()


def _unpack_bits(buf: bytes, bits: int, n: int) -> np.ndarray:
    arr = np.frombuffer(buf, dtype=np.uint8)
    if bits in (1, 2, 4, 8):
        per = 8 // bits
        shifts = (np.arange(per, dtype=np.uint8) * bits)
        return ((arr[:, None] >> shifts) & np.uint8((1 << bits) - 1)).reshape(-1)[:n].astype(np.uint8)
    stream = np.unpackbits(arr, bitorder="little", count=n * bits).reshape(n, bits)
    weights = (1 << np.arange(bits, dtype=np.uint8)).astype(np.uint8)
    return (stream * weights).sum(axis=1, dtype=np.uint8)


def bitpack_header(bits: int, count: int) -> bytes:
    return (BITPACK_MAGIC.to_bytes(4, "little") + bytes([bits, 0, 0, 0]) + int(count).to_bytes(8, "little"))


def cpu_encode_frame(k: torch.Tensor, v: torch.Tensor, spec: FrameSpec, order: torch.Tensor,
                     signs: torch.Tensor, layer: int = 0, seq: int = 1) -> bytearray:
    """Reference encoder: ``k``/``v`` ``[T, H, D]`` (any float dtype),
    ``order`` section-ordered head ids, ``signs`` ``[H, D]`` ±1."""
    T, H, D = spec.T, spec.H, spec.D
    lay = frame_layout(spec)
    buf = bytearray(lay.frame_bytes)
    hdr = np.zeros(16, dtype=np.uint32)
    hdr[:8] = [FRAME_MAGIC, 1, layer, T, H, D, spec.n_low, seq]
    hdr[10] = int(spec.transform)
    hb = bytearray(hdr.tobytes())
    hb[32:36] = bytes([spec.bits[0][0], spec.bits[0][1], spec.bits[1][0], spec.bits[1][1]])
    hb[36:40] = bytes([spec.levels[0][0] - 1, spec.levels[0][1] - 1, spec.levels[1][0] - 1, spec.levels[1][1] - 1])
    buf[0:64] = hb
    Hm = hadamard_matrix(D) / math.sqrt(D) if spec.transform else torch.eye(D)
    if not spec.transform:
        signs = torch.ones_like(signs)
    order_l = [int(x) for x in order.tolist()]
    sec_heads = [order_l[:spec.n_low], order_l[spec.n_low:]]
    for p, x in enumerate((k, v)):
        xf = x.to(torch.float32)
        y = (xf * signs[None].to(torch.float32)) @ Hm  # Hm symmetric
        for s in range(2):
            heads = sec_heads[s]
            if not heads:
                continue
            b = spec.bits[p][s]
            xs = x[:, heads, :]
            off = lay.payload[p][s]
            if b == RAW_BITS:
                raw = xs.to(torch.bfloat16).contiguous().view(torch.int16).numpy().tobytes()
                buf[off:off + len(raw)] = raw
                continue
            lv = spec.levels[p][s]
            ys = y[:, heads, :]
            if p == 0:  # per channel over tokens
                mn = _bf16(ys.amin(dim=0))
                mx = ys.amax(dim=0)
                sc = _bf16(torch.clamp(mx - mn, min=1e-5) / (lv - 1))
                q = torch.clamp(torch.round((ys - mn[None]) * (1.0 / sc)[None]), 0, lv - 1)
                # K aux: full [H*D] arrays in section order
                base = 0 if s == 0 else spec.n_low
                kmin = np.frombuffer(buf, dtype=np.uint16, count=2 * H * D, offset=lay.k_aux).copy()
                mn16 = mn.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16).reshape(-1)
                sc16 = sc.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16).reshape(-1)
                kmin[base * D: base * D + mn16.size] = mn16
                kmin[H * D + base * D: H * D + base * D + sc16.size] = sc16
                buf[lay.k_aux:lay.k_aux + 4 * H * D] = kmin.tobytes()
            else:  # per token over the section
                flat = ys.reshape(T, -1)
                mn = _bf16(flat.amin(dim=1))
                mx = flat.amax(dim=1)
                sc = _bf16(torch.clamp(mx - mn, min=1e-5) / (lv - 1))
                q = torch.clamp(torch.round((flat - mn[:, None]) * (1.0 / sc)[:, None]), 0, lv - 1)
                aux = np.concatenate([
                    mn.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16),
                    sc.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)])
                buf[lay.v_aux[s]:lay.v_aux[s] + aux.nbytes] = aux.tobytes()
            sym = q.to(torch.uint8).numpy().reshape(-1)
            buf[off:off + 16] = bitpack_header(b, sym.size)
            packed = _pack_bits(sym, b)
            buf[off + 16:off + 16 + len(packed)] = packed
    return buf


def cpu_decode_frame(buf: bytes, spec: FrameSpec, order: torch.Tensor, signs: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Reference decoder -> (k, v) bf16 ``[T, H, D]`` in original head order."""
    T, H, D = spec.T, spec.H, spec.D
    lay = frame_layout(spec)
    Hm = hadamard_matrix(D) / math.sqrt(D) if spec.transform else torch.eye(D)
    if not spec.transform:
        signs = torch.ones_like(signs)
    order_l = [int(x) for x in order.tolist()]
    sec_heads = [order_l[:spec.n_low], order_l[spec.n_low:]]
    outs = []
    kaux = None
    if any(spec.section_heads(s) > 0 and spec.bits[0][s] != RAW_BITS for s in range(2)):
        kaux = torch.from_numpy(np.frombuffer(bytes(buf[lay.k_aux:lay.k_aux + 4 * H * D]), dtype=np.int16).copy()
                                ).view(torch.bfloat16).to(torch.float32)
    for p in range(2):
        out = torch.zeros((T, H, D), dtype=torch.float32)
        for s in range(2):
            heads = sec_heads[s]
            if not heads:
                continue
            b = spec.bits[p][s]
            hs = len(heads)
            off = lay.payload[p][s]
            if b == RAW_BITS:
                raw = np.frombuffer(bytes(buf[off:off + T * hs * D * 2]), dtype=np.int16).copy()
                out[:, heads, :] = torch.from_numpy(raw).view(torch.bfloat16).to(torch.float32).reshape(T, hs, D)
                continue
            n = T * hs * D
            sym = _unpack_bits(bytes(buf[off + 16: off + 16 + (n * b + 7) // 8]), b, n)
            q = torch.from_numpy(sym.astype(np.float32)).reshape(T, hs, D)
            if p == 0:
                base = 0 if s == 0 else spec.n_low
                mn = kaux[base * D:(base + hs) * D].reshape(hs, D)
                sc = kaux[H * D + base * D: H * D + (base + hs) * D].reshape(hs, D)
                y = mn[None] + q * sc[None]
            else:
                aux = torch.from_numpy(np.frombuffer(bytes(buf[lay.v_aux[s]:lay.v_aux[s] + 4 * T]), dtype=np.int16).copy()
                                       ).view(torch.bfloat16).to(torch.float32)
                mn, sc = aux[:T], aux[T:]
                y = mn[:, None, None] + q * sc[:, None, None]
            x = (y @ Hm) * signs[heads][None].to(torch.float32)
            out[:, heads, :] = x
        outs.append(out.to(torch.bfloat16))
    return outs[0], outs[1]


# ----------------------------------------------------------------------------
# GPU front-end
# ----------------------------------------------------------------------------

@dataclass
class EncoderState:
    """Per-stream scratch of the encoder: statistics, completion counter and
    (``counter[1]``) the tensor-core path's error word.

    ``stats`` holds the per-channel K statistics ``[min(H*D) | max(H*D)]``
    and, for the tensor-core path (head_dim 128), the per-token V statistics
    ``[section][min(T) | max(T)]`` after them, all as ordered uint32.  The
    last CTA of every layer restores the identities; :meth:`prepare` sets
    them when the geometry changes.  Size it for ``max_tokens`` up front so
    the buffer is never reallocated while a launch may still use it."""

    device: torch.device
    max_hd: int = 2048
    max_tokens: int = 0
    stats: torch.Tensor = field(init=False)
    counter: torch.Tensor = field(init=False)

    def __post_init__(self):
        self.stats = torch.zeros(2 * self.max_hd + 4 * self.max_tokens, dtype=torch.int32, device=self.device)
        self.counter = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._geom = None

    def prepare(self, hd: int, tokens: int = 0) -> None:
        if hd > self.max_hd:
            raise ValueError("H*D exceeds the encoder scratch")
        need = 2 * self.max_hd + 4 * tokens
        if need > self.stats.numel():
            # grow (previous launches on any stream must be done with the old buffer)
            torch.cuda.synchronize(self.device)
            self.stats = torch.zeros(need, dtype=torch.int32, device=self.device)
            self.max_tokens = tokens
            self._geom = None
        if self._geom != (hd, tokens):
            st = self.stats
            st[:hd].fill_(-1)        # 0xFFFFFFFF: min identity
            st[hd:2 * hd].fill_(0)   # 0x00000000: max identity
            v = st[2 * hd:2 * hd + 4 * tokens].view(2, 2, max(tokens, 0))
            v[:, 0].fill_(-1)
            v[:, 1].fill_(0)
            self._geom = (hd, tokens)

    def signed_table(self, sign_bits: torch.Tensor) -> torch.Tensor:
        """Signed Hadamard table of the heads of ``sign_bits`` (head_dim 128),
        built once per sign tensor."""
        key = (sign_bits.data_ptr(), tuple(sign_bits.shape))
        if getattr(self, "_table_key", None) != key:
            from ._ext import ext
            from . import count_launches
            count_launches(1)
            self._table = ext().kv_signed_hadamard(sign_bits.contiguous().view(-1, 4))
            self._table_key = key
        return self._table


def default_tile_tokens(H: int, D: int) -> int:
    """Tokens per CTA tile: one unrolled step of the kernels' row loop
    (8 warps x 32/(D/8) rows x 4 rows per lane = 64 rows for D=128)."""
    rows = 8 * (32 // (D // 8)) * 4
    return max(1, rows // H)


_MMA_ENCODE = os.environ.get("KVSERVE_MMA_ENCODE", "1").strip().lower() not in {"0", "false", "no", "off"}


def encode_layer(k: torch.Tensor, v: torch.Tensor, spec: FrameSpec, order: torch.Tensor,
                 sign_bits: torch.Tensor, frame_ptr: int, state: EncoderState, flag_ptr: int = 0,
                 seq: int = 1, layer: int = 0, pacing: Optional[torch.Tensor] = None,
                 rate_bytes_per_ns: float = 0.0, max_ctas: int = 222, tile_tokens: Optional[int] = None,
                 part_mask: int = 3, block_table: Optional[torch.Tensor] = None, hnd: bool = False,
                 allow_mma: Optional[bool] = None, hs_table: Optional[torch.Tensor] = None,
                 hs_row0: int = 0, trace_ptr: int = 0) -> None:
    """Launch the fused encode of one layer into ``frame_ptr`` (local or peer).

    The defaults (222 CTAs per part; tiles of 64 rows = 64/H tokens, one
    unrolled step of the row loop) give three resident CTAs per SM for the K
    and V parts together and an even tile split.

    ``k``/``v`` are ``[T, H, D]`` views, or — with ``block_table`` — paged
    per-layer caches ``[num_blocks, block_size, H, D]`` (``hnd``: ``[num_blocks,
    H, block_size, D]``) read through the block table (fused gather).
    ``part_mask`` selects K (1), V (2) or both (3).  With head_dim 128, the
    transform on, no raw section and a contiguous ``[T, H, 128]`` source the
    transform runs on the tensor cores (``allow_mma=False`` keeps the
    register butterfly; None follows ``KVSERVE_MMA_ENCODE``, default on),
    with the signed transform table ``hs_table`` (rows of head h of this
    layer at ``(hs_row0 + h) * 128``; built from ``sign_bits`` and cached in
    ``state`` when not given).  Either way there are two launches:
    statistics, then quantise + pack + publish.  ``trace_ptr`` (8-byte
    aligned device address, 0 = off) receives this layer's encode-start and
    frame-published %globaltimer stamps (words 0 and 1 of its four)."""
    if allow_mma is None:
        allow_mma = _MMA_ENCODE
    from ._ext import ext
    from . import count_launches
    active = [(p, s) for p in range(2) for s in range(2) if (part_mask >> p) & 1 and spec.section_heads(s)]
    mma = (allow_mma and spec.D == 128 and spec.transform and spec.T > 0 and spec.H * spec.D <= 1024
           and block_table is None and k.dim() == 3 and k.stride(1) == spec.D and v.stride(1) == spec.D
           and all(spec.bits[p][s] != RAW_BITS for p, s in active))
    if mma and hs_table is None:
        hs_table, hs_row0 = state.signed_table(sign_bits), 0
    count_launches(2 if mma or ((part_mask & 1) and any(spec.section_heads(s) and spec.bits[0][s] != RAW_BITS
                                                         for s in range(2))) else 1)
    state.prepare(spec.H * spec.D, spec.T)
    if tile_tokens is None:
        tile_tokens = default_tile_tokens(spec.H, spec.D)
    ext().kv_encode_layer(k, v, spec.params(), order, sign_bits, int(frame_ptr), state.stats, state.counter,
                          int(flag_ptr), int(seq), int(layer), pacing, float(rate_bytes_per_ns), int(max_ctas),
                          int(tile_tokens), int(part_mask), block_table, bool(hnd), bool(mma), hs_table,
                          int(hs_row0), int(trace_ptr))


def decode_layers(frame_base: int, frame_stride: int, spec: FrameSpec, orders: torch.Tensor,
                  sign_bits: torch.Tensor, kv_cache: torch.Tensor, block_table: torch.Tensor,
                  status: torch.Tensor, tok_offset: int = 0, flags_ptr: int = 0, seq: int = 1,
                  layer_begin: int = 0, num_layers: int = 1, timeout_ns: int = 5_000_000_000,
                  max_ctas: int = 222, tile_tokens: Optional[int] = None, n_lows: Optional[torch.Tensor] = None,
                  part_mask: int = 3, layer_ptrs: Optional[torch.Tensor] = None, hnd: bool = False,
                  trace_ptr: int = 0) -> None:
    """Launch the fused decode of ``num_layers`` consecutive frames into the
    paged cache ``kv_cache`` ``[L, 2, num_blocks, block_size, H, D]``.  With
    ``flags_ptr`` the kernel waits (bounded by ``timeout_ns``) for each
    layer's publish flag to reach ``seq``.  ``n_lows`` (int32 [L] on the
    device) gives each layer's low-section head count when it varies; the
    frame stride must then hold the largest frame.  ``trace_ptr`` (0 = off)
    is a ``[L_total][4]`` u64 stamp array: words 2 and 3 of layer ``l`` get
    its ingest start and end (%globaltimer)."""
    from ._ext import ext
    from . import count_launches
    count_launches(1)
    if tile_tokens is None:
        tile_tokens = default_tile_tokens(spec.H, spec.D)
    ext().kv_decode_layers(int(frame_base), int(frame_stride), spec.params(), orders, sign_bits, kv_cache,
                           block_table, int(tok_offset), int(flags_ptr), int(seq), int(layer_begin),
                           int(num_layers), int(timeout_ns), status, int(max_ctas), int(tile_tokens), n_lows,
                           int(part_mask), layer_ptrs, bool(hnd), int(trace_ptr))
