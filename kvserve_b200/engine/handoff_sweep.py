"""Fused KV hand-off sweep across GPU pairs: compress + P2P push and pull +
decompress into paged blocks, against NCCL send/recv of the same bf16 KV.

    python -m torch.distributed.run --nnodes 1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P -m kvserve_b200.engine.handoff_sweep [--tokens 1024,8192,32768,131072] \\
        [--head-dims 64,128] [--bits 2,3,4,8] [--layers 4] [--iters 5]

N = 2, 4 or 8 gives 1, 2 or 4 prefill->decode pairs (rank i sends to rank
i + N/2, all pairs at once).  Per case every pair moves ``layers`` layers of
one request's KV (8 KV heads); the timed region on every rank runs from a
barrier to the end of its own work (the decode rank: KV in the paged cache),
CUDA events, max over ranks, mean over ``iters`` repetitions.  The product
path is the engine's: one fused encode launch per layer storing the packed
frame into the decode GPU's receive slot with a release flag, one
persistent decode launch acquire-waiting per layer.  The baseline is
``torch.distributed`` NCCL ``isend``/``irecv`` of the raw bf16 K/V of all
layers (no compression, no scatter into blocks).  Roofline of the fused
path: max(bytes through HBM / measured copy bandwidth, packed bytes /
770 GB/s per direction).  Rank 0 prints one JSON object.
"""
from __future__ import annotations

import argparse
import json
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops
from ..ops.microbench import peaks
from ..parallel.context import init_parallel
from ..transport.p2p import FrameReceiver, FrameSender
from .kv_cache import PagedKVCache
from .transfer import KVTransfer, TransferProfile

NVLINK_GBS = 770.0
HEADS = 8
BITS = {2: (4, 4), 3: (8, 8), 4: (16, 16), 8: (256, 256)}


def _profile(bits: Optional[int]) -> TransferProfile:
    if bits is None:
        return TransferProfile.raw()
    lv = BITS[bits]
    return TransferProfile(compressed=True, hybrid_ratio=0.0, key_levels=lv, value_levels=lv)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="1024,8192,32768,131072")
    ap.add_argument("--head-dims", default="64,128")
    ap.add_argument("--bits", default="2,3,4,8")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--iters", type=int, default=5)
    a = ap.parse_args(argv)
    ctx = init_parallel("nccl", timeout_s=120)
    w, rank = ctx.world_size, ctx.rank
    if w < 2 or w % 2:
        raise SystemExit("run with an even number of ranks >= 2")
    dev = torch.device("cuda", torch.cuda.current_device())
    half = w // 2
    sender_side = rank < half
    peer = rank + half if sender_side else rank - half
    L, bs = a.layers, 16
    pk = peaks()
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    tbar = torch.zeros(1, device=dev)
    results = {"world": w, "pairs": half, "layers": L, "kv_heads": HEADS, "peaks": pk, "cases": {}}
    seq = 0

    def timed(fn) -> float:
        nonlocal seq
        ts = []
        for it in range(a.iters + 2):
            seq += 1
            dist.all_reduce(tbar)
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn(seq)
            e.record()
            torch.cuda.synchronize()
            if it >= 2:
                ts.append(s.elapsed_time(e))
        t = torch.tensor([sum(ts) / len(ts)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for D in (int(x) for x in a.head_dims.split(",")):
        for T in (int(x) for x in a.tokens.split(",")):
            g = torch.Generator(device=dev).manual_seed(rank)
            k = torch.randn((L, T, HEADS, D), device=dev, dtype=torch.bfloat16, generator=g)
            v = torch.randn((L, T, HEADS, D), device=dev, dtype=torch.bfloat16, generator=g)
            raw_bytes = 2 * L * T * HEADS * D * 2
            # baseline: NCCL send/recv of the raw KV
            buf = torch.empty_like(k) if not sender_side else None
            bufv = torch.empty_like(v) if not sender_side else None

            def nccl(_s):
                if sender_side:
                    reqs = [dist.isend(k, peer), dist.isend(v, peer)]
                else:
                    reqs = [dist.irecv(buf, peer), dist.irecv(bufv, peer)]
                for r in reqs:
                    r.wait()

            case = {"raw_bytes": raw_bytes, "nccl_ms": round(timed(nccl), 4)}
            case["nccl_GBps"] = round(raw_bytes / case["nccl_ms"] / 1e6, 1)
            del buf, bufv
            nblk = (T + bs - 1) // bs
            for bits in [None] + [int(x) for x in a.bits.split(",") if x]:
                xfer = KVTransfer(_profile(bits), L, HEADS, HEADS, D, 0, 1, dev, T)
                recv = FrameReceiver(L, xfer.frame_stride, 1, dev) if not sender_side else None
                allh = [None] * w
                dist.all_gather_object(allh, recv.handles() if recv is not None else None, group=ctx.cpu_group)
                send = FrameSender(handles=allh[peer], device=dev) if sender_side else None
                cache = PagedKVCache(L, nblk + 1, bs, HEADS, D, dev) if not sender_side else None
                if cache is not None:
                    blocks = cache.allocate(T)
                    table = cache.block_table(blocks, nblk)

                def fused(s):
                    if sender_side:
                        for l in range(L):
                            xfer.encode(l, k[l], v[l], send.frame_ptr(0, l), send.flag_ptr(0, l), s)
                    else:
                        xfer.ingest_all(T, recv.slot_base(0), recv.frame_stride, recv.flags_base(0), cache.cache,
                                        table, status, s, int(10e9))

                t = timed(fused)
                ops.check_device_status(dev)
                if int(status[0].item()) != 0:
                    raise RuntimeError(f"hand-off status {int(status[0].item())}")
                packed = xfer.payload_bytes(T)
                hbm = raw_bytes + packed        # read bf16 + write frame (decode: read frame + write bf16)
                roof = max(hbm / (pk["hbm_gbs"] * 1e6), packed / (NVLINK_GBS * 1e6))
                name = "raw" if bits is None else f"{bits}bit"
                case[name] = {"ms": round(t, 4), "ratio": round(raw_bytes / packed, 3),
                              "speedup_vs_nccl": round(case["nccl_ms"] / t, 2),
                              "frac_of_roofline": round(roof / t, 3)}
                torch.cuda.synchronize()
                dist.barrier(group=ctx.cpu_group)
                if send is not None:
                    send.close()
                if recv is not None:
                    recv.close()
                del cache
            results["cases"][f"D{D}_T{T}"] = case
            del k, v
            torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(results))
    torch.cuda.synchronize()
    dist.barrier(group=ctx.cpu_group)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
