"""Compression component speeds on the GPU: this framework's fused kernels
next to PyTorch restatements of two published KV-cache compressors.

The reference times each component of its search space — and KIVI,
CacheGen, nvCOMP ANS/Bitcomp and torchac — on real prompts and writes one
CSV per model (kvserve_v1/offline_search/evaluation/component_speed/*.py,
columns ``type,input_length,original_size(GB),prefill_time(s),
decode_time(s),prefill_throughput(GB/s),decode_throughput(GB/s)``).  Here
the KV is synthetic with the benchmark's distribution (values N(0,1), keys
N(0,1) with 4 outlier channels per head scaled x8) and the rows are:

* ``kvserve-fused-k4v2`` / ``-k4v4`` / ``-k8v8``: the fused frame encode
  (Hadamard + min-max quantisation + bit packing, one layer per call) and
  the fused decode into a paged cache — the product hot path;
* ``hadamard``: the random-sign Hadamard rows kernel alone;
* ``lossless``: the kvs-rze-v1 codec on a 4-bit packed payload;
* ``kivi-2bit`` / ``kivi-4bit``: KIVI's asymmetric group quantisation (keys
  grouped along tokens per channel, values grouped along channels per
  token, group 32) with the integer codes packed into 32-bit words, in
  plain PyTorch (no KIVI kernels are installed here);
* ``cachegen-style``: CacheGen's idea — anchor token per chunk, deltas of
  the others to it, per-channel quantisation of the deltas — followed by
  this repository's lossless codec in place of its arithmetic coder.

Compress = ``prefill_time``, decompress = ``decode_time`` (the reference's
names); throughputs are raw bf16 bytes / time.

    python -m kvserve_b200.offline_search.component_speed --model llama-3.1-8b \\
        --lengths 1024,4096,16384 --out speeds.csv
"""
from __future__ import annotations

import argparse
import csv
import math
from typing import Callable

import torch

from ..engine.serving import synthetic_kv

COLUMNS = ["type", "input_length", "original_size(GB)", "prefill_time(s)", "decode_time(s)",
           "prefill_throughput(GB/s)", "decode_throughput(GB/s)"]


def _time_s(fn: Callable[[], None], iters: int = 10) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters / 1e3


# ------------------------------------------------------------ KIVI (PyTorch)
def kivi_compress(x: torch.Tensor, bits: int, per_channel: bool, group: int = 32):
    """x [T, H, D] -> (packed int32 codes, min, scale).  ``per_channel``:
    groups of ``group`` tokens per (head, channel) (KIVI's keys); otherwise
    groups of ``group`` channels per (token, head) (its values)."""
    T, H, D = x.shape
    xf = x.float()
    if per_channel:
        Tg = T // group * group
        g = xf[:Tg].reshape(Tg // group, group, H, D)
        red = 1
    else:
        g = xf.reshape(T, H, D // group, group)
        red = 3
    mn = g.amin(dim=red, keepdim=True)
    sc = (g.amax(dim=red, keepdim=True) - mn).clamp_min(1e-5) / (2 ** bits - 1)
    q = ((g - mn) / sc).round_().clamp_(0, 2 ** bits - 1).to(torch.int32).reshape(-1)
    per = 32 // bits
    q = q[: q.numel() // per * per].view(-1, per)
    shifts = torch.arange(0, 32, bits, device=x.device, dtype=torch.int32)
    packed = (q << shifts).sum(dim=1, dtype=torch.int32)
    return packed, mn.to(torch.bfloat16), sc.to(torch.bfloat16)


def kivi_decompress(packed: torch.Tensor, mn: torch.Tensor, sc: torch.Tensor, bits: int, per_channel: bool,
                    group: int = 32) -> torch.Tensor:
    """Inverse of :func:`kivi_compress` (grouped layout: [T/g, g, H, D] for
    keys, [T, H, D/g, g] for values)."""
    shifts = torch.arange(0, 32, bits, device=packed.device, dtype=torch.int32)
    q = ((packed.unsqueeze(1) >> shifts) & (2 ** bits - 1)).reshape(-1)
    shape = list(mn.shape)
    shape[1 if per_channel else 3] = group
    n = math.prod(shape)
    return (q[:n].view(shape).float() * sc.float() + mn.float()).to(torch.bfloat16)


# ------------------------------------------------- CacheGen-style (PyTorch)
def cachegen_compress(x: torch.Tensor, bits: int = 4, chunk: int = 16):
    """x [T, H, D]: per chunk of ``chunk`` tokens the first token is kept in
    bf16 (anchor) and the others become deltas to it, quantised per (head,
    channel) over the chunk with ``bits`` bits; the byte codes then go
    through the lossless codec.  Returns (payload, anchors, min, scale)."""
    from ..ops.lossless import gpu_encode
    T, H, D = x.shape
    Tc = T // chunk * chunk
    g = x[:Tc].float().view(Tc // chunk, chunk, H, D)
    anchor = g[:, :1]
    d = g[:, 1:] - anchor
    mn = d.amin(dim=1, keepdim=True)
    sc = (d.amax(dim=1, keepdim=True) - mn).clamp_min(1e-5) / (2 ** bits - 1)
    q = ((d - mn) / sc).round_().clamp_(0, 2 ** bits - 1).to(torch.uint8).contiguous()
    return gpu_encode(q.view(-1)), anchor.to(torch.bfloat16), mn.to(torch.bfloat16), sc.to(torch.bfloat16)


def cachegen_decompress(payload: torch.Tensor, anchor: torch.Tensor, mn: torch.Tensor, sc: torch.Tensor,
                        chunk: int = 16) -> torch.Tensor:
    from ..ops.lossless import gpu_decode
    n, _, H, D = anchor.shape
    q = gpu_decode(payload).view(n, chunk - 1, H, D).float()
    d = q * sc.float() + mn.float()
    return torch.cat([anchor.float(), anchor.float() + d], dim=1).reshape(n * chunk, H, D).to(torch.bfloat16)


# ----------------------------------------------------------------- harness
def measure(model: str, lengths: list[int], iters: int = 10) -> list[dict]:
    """Rows of the component-speed table for one model's per-GPU KV shape
    (all KV heads of one layer; times are per layer)."""
    from ..engine.kv_cache import PagedKVCache
    from ..engine.serving import ENGINE_PROFILES
    from ..engine.transfer import KVTransfer
    from ..models.config import get_config
    from ..ops import ext
    from ..ops.lossless import gpu_decode, gpu_encode
    from ..transport.p2p import FrameReceiver, FrameSender
    cfg = get_config(model)
    H, D = cfg.num_kv_heads, cfg.head_dim
    dev = torch.device("cuda")
    rows = []

    def row(name, T, comp, decomp):
        raw = 2 * T * H * D * 2
        tc, td = _time_s(comp, iters), _time_s(decomp, iters)
        rows.append({"type": name, "input_length": T, "original_size(GB)": round(raw / 1e9, 6),
                     "prefill_time(s)": round(tc, 7), "decode_time(s)": round(td, 7),
                     "prefill_throughput(GB/s)": round(raw / tc / 1e9, 2),
                     "decode_throughput(GB/s)": round(raw / td / 1e9, 2)})

    for T in lengths:
        kv = synthetic_kv(T, H, D, seed=0)[0, :, 0].to(dev)   # [2, T, H, D]
        k, v = kv[0].contiguous(), kv[1].contiguous()
        for name in ("k4v2", "k4v4", "k8v8"):
            x = KVTransfer(ENGINE_PROFILES[name], 1, H, H, D, 0, 1, dev, T)
            rcv = FrameReceiver(1, x.frame_stride, 1, dev)
            snd = FrameSender(local=rcv, device=dev)
            cache = PagedKVCache(1, T // 16 + 2, 16, H, D, dev)
            table = cache.block_table(cache.allocate(T), T // 16 + 2)
            status = torch.zeros(1, dtype=torch.int32, device=dev)
            row(f"kvserve-fused-{name}", T, lambda: x.encode(0, k, v, snd.frame_ptr(0, 0), 0, 1),
                lambda: x.ingest_layer(0, T, snd.frame_ptr(0, 0), cache.cache, table, status, 1))
            torch.cuda.synchronize()
            rcv.close()
        rows_h = k.view(-1, D)
        out_h = torch.empty_like(rows_h)
        signs = (torch.randint(0, 2, (D,), device=dev) * 2 - 1).float()
        row("hadamard", T, lambda: ext().fwht_rows(rows_h, out_h, signs, False),
            lambda: ext().fwht_rows(out_h, rows_h, signs, True))
        packed = torch.randint(0, 256, (T * H * D,), dtype=torch.uint8, device=dev) & 0x77
        enc = gpu_encode(packed)
        row("lossless", T, lambda: gpu_encode(packed), lambda: gpu_decode(enc))
        for bits in (2, 4):
            ck, cv = kivi_compress(k, bits, True), kivi_compress(v, bits, False)
            row(f"kivi-{bits}bit", T, lambda: (kivi_compress(k, bits, True), kivi_compress(v, bits, False)),
                lambda: (kivi_decompress(*ck, bits, True), kivi_decompress(*cv, bits, False)))
        ckv = [cachegen_compress(t) for t in (k, v)]
        row("cachegen-style", T, lambda: [cachegen_compress(t) for t in (k, v)],
            lambda: [cachegen_decompress(*c) for c in ckv])
    return rows


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--lengths", default="1024,4096,16384")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    rows = measure(a.model, [int(x) for x in a.lengths.split(",") if x], a.iters)
    if a.out:
        with open(a.out, "w", newline="") as f:
            w = csv.DictWriter(f, fieldnames=COLUMNS)
            w.writeheader()
            w.writerows(rows)
    for r in rows:
        print(",".join(str(r[c]) for c in COLUMNS))


if __name__ == "__main__":
    main()
