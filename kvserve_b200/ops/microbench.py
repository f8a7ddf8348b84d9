"""Kernel microbenchmarks of the sm_100a library (one GPU).

    python -m kvserve_b200.ops.microbench [--case all|gemm|gemv|flash|decode|handoff|lossless|norm]
                                          [--iters N] [--quick] [--once]

Every number is a CUDA-event time on the launching stream after warm-up,
with a synchronise on both sides; decode-size kernels (GEMV, paged decode)
and the per-layer hand-off kernels are timed as a CUDA-graph replay of many
calls (the way a decode step runs, and so that the wrappers' host work is
not what is measured).  Working sets are larger than L2 (126 MB)
or rotated across buffers whose total is, so DRAM figures are honest;
``--once`` runs each kernel a single time after three warm-ups (the mode to
run under a profiler, whose numbers are never reported as timings).
Fractions are against the measured peaks of ``MEASURED_PEAKS.json`` at the
repository root when present (``hbm_gbs``, ``bf16_tflops``), else the
fallbacks 6650 GB/s and 1590 TFLOP/s.
"""
from __future__ import annotations

import argparse
import json
import math
import os
from typing import Callable, Sequence

import torch

from . import (flash_prefill, gemm, gemm_qkv_rope, gemm_silu, gemv, interleave_gate_up, paged_decode_attention,
               rmsnorm, rope_qkv, silu_mul)
from . import kv_codec as kc
from .lossless import gpu_decode, gpu_encode

L2_BYTES = 126 * 2 ** 20


def peaks() -> dict:
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    out = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained"):
            if isinstance(d.get(k), (int, float)):
                out[k] = float(d[k])
        out["source"] = "measured"
    return out


def time_ms(fns: list[Callable[[], None]], iters: int, once: bool = False) -> float:
    """Mean ms per call, cycling through ``fns`` (distinct buffers)."""
    for i in range(3):
        fns[i % len(fns)]()
    torch.cuda.synchronize()
    n = 1 if once else iters
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(n):
        fns[i % len(fns)]()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / n


def time_graph_ms(fns: list[Callable[[], None]], iters: int) -> float:
    """Mean ms per call of ``iters`` calls captured in one CUDA graph (the
    way the decode step runs them), so host launch overhead is excluded."""
    for i in range(3):
        fns[i % len(fns)]()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(iters):
            fns[i % len(fns)]()
    torch.cuda.synchronize()
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    g.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def copies_for(bytes_per_call: int) -> int:
    return max(1, math.ceil(2 * L2_BYTES / max(1, bytes_per_call)))


def case_gemm(a, pk):
    shapes = [(8192, 6144, 4096), (8192, 4096, 4096), (8192, 28672, 4096), (8192, 4096, 14336)]
    if not a.quick:
        shapes += [(4096, 4096, 4096), (8192, 8192, 8192)]
    res = {}
    for M, N, K in shapes:
        A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
        C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        t = time_ms([lambda: gemm(A, B, C)], a.iters, a.once)
        r = {"ms": round(t, 4), "tflops": round(2 * M * N * K / t / 1e9, 1)}
        r["frac_of_measured_bf16"] = round(r["tflops"] / pk["bf16_tflops"], 3)
        if not a.once:
            tc = time_ms([lambda: torch.matmul(A, B.T, out=C)], a.iters)
            r["cublas_tflops"] = round(2 * M * N * K / tc / 1e9, 1)
        res[f"gemm_{M}x{N}x{K}"] = r
    # gate/up projection with the SiLU-mul epilogue (output [M, N/2])
    M, I, K = 8192, 14336, 4096
    A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    # unit-variance pre-activations, as after an RMSNorm-ed input
    W = interleave_gate_up(torch.randn(I, K, device="cuda", dtype=torch.bfloat16) / math.sqrt(K),
                           torch.randn(I, K, device="cuda", dtype=torch.bfloat16) / math.sqrt(K))
    Y = torch.empty(M, I, device="cuda", dtype=torch.bfloat16)
    t = time_ms([lambda: gemm_silu(A, W, Y)], a.iters, a.once)
    res[f"gemm_silu_{M}x{2 * I}x{K}"] = {"ms": round(t, 4), "tflops": round(2 * M * 2 * I * K / t / 1e9, 1),
                                         "frac_of_measured_bf16": round(2 * M * 2 * I * K / t / 1e9
                                                                        / pk["bf16_tflops"], 3)}
    # QKV projection with bias-free rotary epilogue and K/V copies (Llama-3.1-8B shape)
    Hq, Hkv, K = 32, 8, 4096
    N = (Hq + 2 * Hkv) * 128
    W = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / math.sqrt(K)
    Y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    pos = torch.arange(M, device="cuda", dtype=torch.int32)
    inv = 1.0 / (500000.0 ** (torch.arange(0, 128, 2, device="cuda").float() / 128))
    ang = pos.float()[:, None] * inv[None]
    cs = torch.cat([ang.cos(), ang.sin()], -1).contiguous()
    kd = torch.empty(M, Hkv, 128, device="cuda", dtype=torch.bfloat16)
    vd = torch.empty_like(kd)
    t = time_ms([lambda: gemm_qkv_rope(A, W, Hq, Hkv, pos, cs, k_dst=kd, v_dst=vd, out=Y)], a.iters, a.once)
    res[f"gemm_qkv_rope_{M}x{N}x{K}"] = {"ms": round(t, 4), "tflops": round(2 * M * N * K / t / 1e9, 1),
                                         "frac_of_measured_bf16": round(2 * M * N * K / t / 1e9 / pk["bf16_tflops"],
                                                                        3)}
    return res


def case_gemv(a, pk):
    res = {}
    # M = 1 on the 8B shapes; M = 1/4/8 on the 70B TP4 shapes a batched decode step runs
    shapes = [(1, 6144, 4096), (1, 4096, 4096), (1, 28672, 4096), (1, 4096, 14336), (1, 128256, 4096)]
    shapes += [(m, 14336, 8192) for m in (1, 4, 8)] + [(m, 8192, 7168) for m in (1, 8)]
    for M, N, K in shapes:
        nb = N * K * 2
        ws = [torch.randn(N, K, device="cuda", dtype=torch.bfloat16) for _ in range(copies_for(nb))]
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        fns = [lambda w=w: gemv(x, w, y) for w in ws]
        t = time_ms(fns, a.iters * 4, a.once) if a.once else time_graph_ms(fns, a.iters * 4)
        gbs = nb / t / 1e6
        res[f"gemv_M{M}_{N}x{K}"] = {"ms": round(t, 4), "GBps": round(gbs, 1),
                                     "frac_of_measured_hbm": round(gbs / pk["hbm_gbs"], 3)}
    return res


def case_flash(a, pk):
    res = {}
    for T, Hq, Hkv in [(8192, 32, 8), (4096, 32, 8)] + ([] if a.quick else [(16384, 32, 8), (32768, 28, 4)]):
        qkv = torch.randn(T, (Hq + 2 * Hkv) * 128, device="cuda", dtype=torch.bfloat16)
        out = torch.empty(T, Hq * 128, device="cuda", dtype=torch.bfloat16)
        fl = 4 * T * T * 128 * Hq / 2
        r = {}
        # the default kernel first, then the K-ring and exponential-mix variants
        for name, ks, pm in (("default", 0, 0), ("kstages3", 3, 0), ("poly_11", 2, 0x11),
                             ("poly_55", 2, 0x55), ("poly_ff", 2, 0xFF)):
            t = time_ms([lambda: flash_prefill(qkv, Hq, Hkv, out=out, kstages=ks, poly=pm)], max(3, a.iters // 2),
                        a.once)
            r[name] = {"ms": round(t, 4), "tflops": round(fl / t / 1e9, 1),
                            "frac_of_measured_bf16": round(fl / t / 1e9 / pk["bf16_tflops"], 3)}
            if a.once:
                break
        if not a.once and T <= 16384:
            import torch.nn.functional as F
            q = qkv[:, :Hq * 128].view(T, Hq, 128).transpose(0, 1).unsqueeze(0).contiguous()
            k = qkv[:, Hq * 128:(Hq + Hkv) * 128].view(T, Hkv, 128).transpose(0, 1).unsqueeze(0).contiguous()
            v = qkv[:, (Hq + Hkv) * 128:].view(T, Hkv, 128).transpose(0, 1).unsqueeze(0).contiguous()
            ts = time_ms([lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)],
                         max(3, a.iters // 2))
            r["sdpa_tflops"] = round(fl / ts / 1e9, 1)
        res[f"flash_T{T}_q{Hq}_kv{Hkv}"] = r
    return res


def case_decode(a, pk):
    res = {}
    # Llama-3.1-8B (32 q / 8 KV heads) and Llama-3-70B at TP4 (16 q / 2 KV heads: 8 per KV head)
    for B, ctx, Hq, Hkv in [(1, 8192, 32, 8), (8, 8192, 32, 8), (32, 4096, 32, 8), (1, 16384, 16, 2),
                            (8, 16384, 16, 2)]:
        D, bs = 128, 16
        nblk = B * ctx // bs
        kv_bytes = 2 * nblk * bs * Hkv * D * 2
        sets = []
        for _ in range(copies_for(kv_bytes)):
            kc_ = torch.randn(nblk, bs, Hkv, D, device="cuda", dtype=torch.bfloat16)
            vc_ = torch.randn(nblk, bs, Hkv, D, device="cuda", dtype=torch.bfloat16)
            sets.append((kc_, vc_))
        q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16)
        table = torch.randperm(nblk, device="cuda", dtype=torch.int32).view(B, -1)
        lens = torch.full((B,), ctx, device="cuda", dtype=torch.int32)
        out = torch.empty_like(q)
        fns = [lambda s=s: paged_decode_attention(q, s[0], s[1], table, lens, ctx, out=out) for s in sets]
        t = time_ms(fns, a.iters * 4, a.once) if a.once else time_graph_ms(fns, a.iters * 4)
        gbs = kv_bytes / t / 1e6
        res[f"paged_decode_B{B}_ctx{ctx}_q{Hq}_kv{Hkv}"] = {"ms": round(t, 4), "GBps": round(gbs, 1),
                                              "frac_of_measured_hbm": round(gbs / pk["hbm_gbs"], 3)}
    return res


def case_handoff(a, pk):
    """Fused KV hand-off kernels on one GPU (frames written to local memory):
    compress = Hadamard+quant+bitpack of one layer's K/V into a frame;
    decompress = unpack+dequant+inverse Hadamard into paged blocks."""
    from ..compression.heads import pack_sign_bits, rademacher_signs
    res = {}
    tokens = [1024, 8192, 32768] if a.quick else [1024, 4096, 8192, 32768, 131072]
    if a.tokens:
        tokens = [a.tokens]
    bit_sets = {"k4v2": ((16, 16), (4, 4)), "k8v8": ((256, 256), (256, 256)), "k3v3": ((8, 8), (8, 8)),
                "k2v2": ((4, 4), (4, 4)), "k4v4": ((16, 16), (16, 16))}
    pick = ["k4v2", "k8v8"] if a.quick else list(bit_sets)
    if a.bits:
        pick = [a.bits]
    H = 8
    for D in ((a.head_dim,) if a.head_dim else (128, 64)):
        signs = pack_sign_bits(rademacher_signs(0, 0, H, D)).cuda()
        order = torch.arange(H, dtype=torch.int32, device="cuda")
        for T in tokens:
            raw = 2 * T * H * D * 2
            nset = copies_for(raw)
            ks = [torch.randn(T, H, D, device="cuda", dtype=torch.bfloat16) for _ in range(nset)]
            vs = [torch.randn(T, H, D, device="cuda", dtype=torch.bfloat16) for _ in range(nset)]
            for name in pick:
                kl, vl = bit_sets[name]
                spec = kc.spec_from_profile(T, H, D, 0, kl, vl)
                fb = kc.frame_layout(spec).frame_bytes
                frames = [torch.empty(fb, dtype=torch.uint8, device="cuda") for _ in range(nset)]
                st = kc.EncoderState(torch.device("cuda"))
                enc = [lambda i=i: kc.encode_layer(ks[i], vs[i], spec, order, signs, frames[i].data_ptr(), st)
                       for i in range(nset)]
                # CUDA-graph replay: the per-call Python work of the wrappers
                # would otherwise be what the events measure
                te = time_ms(enc, 1, True) if a.once else time_graph_ms(enc, max(nset, a.iters * 2))
                bs = 16
                nblk = T // bs
                caches = [torch.empty(1, 2, nblk, bs, H, D, device="cuda", dtype=torch.bfloat16)
                          for _ in range(nset)]
                table = torch.arange(nblk, dtype=torch.int32, device="cuda").view(1, -1)
                status = torch.zeros(4, dtype=torch.int32, device="cuda")
                orders = order.view(1, -1)
                signs_l = signs.unsqueeze(0)
                dec = [lambda i=i: kc.decode_layers(frames[i].data_ptr(), fb, spec, orders, signs_l, caches[i],
                                                    table, status) for i in range(nset)]
                td = time_ms(dec, 1, True) if a.once else time_graph_ms(dec, max(nset, a.iters * 2))
                if int(status[0].item()) != 0:
                    raise RuntimeError(f"decode status {int(status[0].item())}")
                moved = raw + fb  # bf16 K/V read (written) + frame written (read)
                res[f"handoff_D{D}_T{T}_{name}"] = {
                    "ratio": round(raw / fb, 3),
                    "compress_ms": round(te, 4), "compress_GBps_raw": round(raw / te / 1e6, 1),
                    "compress_frac_of_measured_hbm": round(moved / te / 1e6 / pk["hbm_gbs"], 3),
                    "decompress_ms": round(td, 4), "decompress_GBps_raw": round(raw / td / 1e6, 1),
                    "decompress_frac_of_measured_hbm": round(moved / td / 1e6 / pk["hbm_gbs"], 3),
                }
                del frames, caches
    return res


def case_lossless(a, pk):
    res = {}
    n = 64 * 2 ** 20
    g = torch.Generator(device="cuda").manual_seed(0)
    # 4-bit symbols stored one per byte: the codec's typical input
    raws = [torch.randint(0, 16, (n,), device="cuda", dtype=torch.uint8, generator=g) for _ in range(4)]
    te = time_ms([lambda r=r: gpu_encode(r) for r in raws], max(3, a.iters // 4), a.once)
    enc = gpu_encode(raws[0])
    td = time_ms([lambda: gpu_decode(enc)], max(3, a.iters // 4), a.once)
    res["lossless_64MiB_4bit_symbols"] = {"ratio": round(n / enc.numel(), 3), "encode_ms": round(te, 4),
                                          "encode_GBps": round(n / te / 1e6, 1), "decode_ms": round(td, 4),
                                          "decode_GBps": round(n / td / 1e6, 1),
                                          "note": "times include the host read of the encoded size"}
    return res


def case_norm(a, pk):
    res = {}
    T, Hd = 8192, 4096
    xs = [torch.randn(T, Hd, device="cuda", dtype=torch.bfloat16) for _ in range(4)]
    rs = [torch.randn(T, Hd, device="cuda", dtype=torch.bfloat16) for _ in range(4)]
    w = torch.randn(Hd, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(T, Hd, device="cuda", dtype=torch.bfloat16)
    t = time_ms([lambda i=i: rmsnorm(xs[i], w, 1e-5, residual=rs[i], out=out) for i in range(4)], a.iters, a.once)
    nb = 4 * T * Hd * 2
    res["rmsnorm_residual_8192x4096"] = {"ms": round(t, 4), "GBps": round(nb / t / 1e6, 1),
                                         "frac_of_measured_hbm": round(nb / t / 1e6 / pk["hbm_gbs"], 3)}
    gu = [torch.randn(T, 2 * 14336, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    o2 = torch.empty(T, 14336, device="cuda", dtype=torch.bfloat16)
    t = time_ms([lambda i=i: silu_mul(gu[i], o2) for i in range(2)], a.iters, a.once)
    nb = 3 * T * 14336 * 2
    res["silu_mul_8192x14336"] = {"ms": round(t, 4), "GBps": round(nb / t / 1e6, 1),
                                  "frac_of_measured_hbm": round(nb / t / 1e6 / pk["hbm_gbs"], 3)}
    Hq, Hkv, D = 32, 8, 128
    qkv = [torch.randn(T, (Hq + 2 * Hkv) * D, device="cuda", dtype=torch.bfloat16) for _ in range(3)]
    pos = torch.arange(T, device="cuda", dtype=torch.int32)
    inv = 1.0 / (500000.0 ** (torch.arange(0, D, 2, device="cuda").float() / D))
    ang = pos.float()[:, None] * inv[None]
    cs = torch.cat([ang.cos(), ang.sin()], -1).contiguous()
    kd = torch.empty(T, Hkv, D, device="cuda", dtype=torch.bfloat16)
    vd = torch.empty(T, Hkv, D, device="cuda", dtype=torch.bfloat16)
    t = time_ms([lambda i=i: rope_qkv(qkv[i], Hq, Hkv, D, pos, cs, kd, vd) for i in range(3)], a.iters, a.once)
    nb = T * (Hq + Hkv) * D * 2 * 2 + T * 2 * Hkv * D * 2 * 2
    res["rope_qkv_8192_q32_kv8"] = {"ms": round(t, 4), "GBps": round(nb / t / 1e6, 1),
                                    "frac_of_measured_hbm": round(nb / t / 1e6 / pk["hbm_gbs"], 3)}
    return res


def link_model(handoff: dict, gbps: Sequence[float] = (20, 50, 100, 200, 400, 7200)) -> dict:
    """Theoretical per-layer hand-off time at several link speeds (the
    reference's codec-throughput tool reports 20/50/100/200 Gbps; 7200 Gbps
    is one NVLink 5 direction): raw = bytes / link; compressed =
    compress + packed bytes / link + decompress (serial, no overlap)."""
    out = {}
    for key, r in handoff.items():
        if not key.startswith("handoff_"):
            continue
        raw_b = r["compress_GBps_raw"] * 1e6 * r["compress_ms"]   # bytes of bf16 K+V
        packed = raw_b / r["ratio"]
        row = {}
        for g in gbps:
            bps = g * 1e9 / 8
            t_raw = 1e3 * raw_b / bps
            t_c = r["compress_ms"] + 1e3 * packed / bps + r["decompress_ms"]
            row[f"{g:g}Gbps"] = {"raw_ms": round(t_raw, 4), "compressed_ms": round(t_c, 4),
                                 "speedup": round(t_raw / t_c, 2)}
        out[key.replace("handoff_", "link_")] = row
    return out


CASES = {"gemm": case_gemm, "gemv": case_gemv, "flash": case_flash, "decode": case_decode,
         "handoff": case_handoff, "lossless": case_lossless, "norm": case_norm}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all", choices=["all", *CASES])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--once", action="store_true")
    ap.add_argument("--tokens", type=int, default=0, help="handoff: only this token count")
    ap.add_argument("--bits", default="", help="handoff: only this bit set (e.g. k4v2)")
    ap.add_argument("--head-dim", type=int, default=0, help="handoff: only this head_dim")
    a = ap.parse_args(argv)
    pk = peaks()
    out = {"peaks": pk}
    from ..utils.clocks import ClockSampler
    sampler = ClockSampler([torch.cuda.current_device()])
    sampler.start()
    try:
        for name, fn in CASES.items():
            if a.case in ("all", name):
                out.update(fn(a, pk))
    finally:
        out["clocks"] = sampler.stop()
    if any(k.startswith("handoff_") for k in out):
        out.update(link_model(out))
    print(json.dumps(out, indent=1))


if __name__ == "__main__":
    main()
