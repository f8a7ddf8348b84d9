"""The CPU configuration of the benchmark suite, end to end: compression of
a synthetic KV sample plus a two-process PD transfer over gloo (role of
the reference's CPU round trip, kvserve_v1/compression/manager.py:54-345 with
kvserve_v1/transport/nccl_transport.py on a CPU data plane).

The sample is ``[layers=2, K/V=2, tokens=256, kv_heads=4, head_dim=128]``
bf16: values N(0,1), keys N(0,1) with 4 fixed outlier channels per head
scaled x8 (seed 0).  The profile is random-sign Hadamard (size 128) ->
min-max (keys 4-bit per channel, values 4-bit per token, split by head) ->
BitPack 4-bit.  The producer process compresses the sample, builds the
:class:`~kvserve_b200.compression.wire.CompressedWire` and sends it as one
bundle through :class:`~kvserve_b200.transport.nccl_transport.NcclTransport`
(``data_plane="gloo"``, ZeroMQ control, byte credits); the consumer process
restores the wire, decompresses and reports the reconstruction error against
the same seeded sample.

    python -m kvserve_b200.engine.config0          # prints one JSON line
"""
from __future__ import annotations

import json
import multiprocessing as mp
import os
import socket
import time

import torch

PROFILE = {
    "enabled": True,
    "pipeline": ["transformer", "quantizer", "codec"],
    "transformer_config": {"transform_type": "hadamard", "seed": 3237919422},
    "quantizer_config": {"model_name": "synthetic", "hybrid_ratio": 0.0, "high_key_max_value": 15,
                         "high_value_max_value": 15, "low_key_max_value": 15, "low_value_max_value": 15,
                         "axis_key": "channel", "axis_value": "token", "split_type": "head",
                         "num_layers": 2, "num_kv_heads": 4},
    "codec_config": {"codec_type": "bitpack", "bitpack_bits": 4},
}
LAYERS, TOKENS, HEADS, DIM = 2, 256, 4, 128


def synthetic_kv(seed: int = 0) -> torch.Tensor:
    """``[L, 2, 1, T, H, D]`` bf16 sample (keys with 4 outlier channels x8)."""
    g = torch.Generator().manual_seed(seed)
    kv = torch.randn((LAYERS, 2, 1, TOKENS, HEADS, DIM), generator=g)
    ch = torch.randperm(DIM, generator=g)[:4]
    kv[:, 0, :, :, :, ch] *= 8
    return kv.to(torch.bfloat16)


def _adapter():
    from ..compression.adapter import KVCompressionAdapter
    return KVCompressionAdapter(PROFILE, num_kv_heads=HEADS, head_size=DIM, num_layers=LAYERS)


def _finish(q, role: str, out: dict, done=None) -> None:
    """Report, then leave without closing the transport: its control thread
    may still be inside a ZeroMQ call, and closing the socket under it aborts
    the process before the report is out."""
    q.put((role, out))
    if done is not None:
        done.wait(60)            # the consumer may still be returning credits
    q.close()
    q.join_thread()
    os._exit(0)


def _producer(port: int, q, done) -> None:
    from ..compression.adapter import add_sentinel
    from ..compression.wire import build_wire
    from ..transport.nccl_transport import NcclTransport
    out = {"error": None}
    try:
        kv = synthetic_kv()
        ad = _adapter()
        ad.compress(kv, "warm-up")                  # first call builds the pipeline
        t0 = time.perf_counter()
        c = ad.compress(kv, "config0")
        out["compress_ms"] = 1e3 * (time.perf_counter() - t0)
        w = build_wire(c, 512 << 20)
        out.update(original_bytes=int(c.original_size), compressed_bytes=int(c.compressed_size),
                   wire_bytes=int(w.nbytes))
        t = NcclTransport(True, "127.0.0.1", port, data_plane="gloo", control_timeout_s=60)
        t0 = time.perf_counter()
        t.send_bundle("config0", add_sentinel([f"layer.{i}" for i in range(LAYERS)]), w.meta, w.body_chunks,
                      w.aux_tensors)
        out["sent"] = bool(t.wait_for_sent(timeout=120))
        out["send_ms"] = 1e3 * (time.perf_counter() - t0)
    except Exception:  # noqa: BLE001 - reported to the parent
        import traceback
        out["error"] = traceback.format_exc()
    _finish(q, "producer", out, done)


def _consumer(port: int, q, done) -> None:
    from ..compression.adapter import is_compressed_layer_names
    from ..compression.wire import CompressedWire, restore_from_wire
    from ..transport.nccl_transport import NcclTransport
    out = {"error": None}
    try:
        t = NcclTransport(False, "127.0.0.1", port, data_plane="gloo", recv_buffer_size=64 << 20)
        deadline = time.time() + 120
        got = None
        while got is None and time.time() < deadline:
            for _, items in t.drain_received().items():
                got = items[0]
            time.sleep(0.005)
        if got is None:
            raise TimeoutError("no payload arrived")
        names, payload = got
        if payload is None or not is_compressed_layer_names(names):
            raise RuntimeError("expected a compressed bundle")
        ad = _adapter()
        wire = CompressedWire(payload["meta"], payload["body_chunks"], payload["aux_tensors"])
        ad.decompress(restore_from_wire(wire))      # first call builds the pipeline
        t0 = time.perf_counter()
        rec = ad.decompress(restore_from_wire(wire))
        out["decompress_ms"] = 1e3 * (time.perf_counter() - t0)
        t.release_received("config0", t.payload_nbytes(payload))
        kv = synthetic_kv().float()
        err = rec.float() - kv
        out["mse"] = float(err.pow(2).mean())
        out["mse_keys"] = float(err[:, 0].pow(2).mean())
        out["mse_values"] = float(err[:, 1].pow(2).mean())
        out["relative_error"] = float(err.norm() / kv.norm())
        out["signal_power"] = float(kv.pow(2).mean())
    except Exception:  # noqa: BLE001 - reported to the parent
        import traceback
        out["error"] = traceback.format_exc()
    _finish(q, "consumer", out)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def run(timeout_s: float = 180.0) -> dict:
    """Run both processes; returns the merged report (``error`` set on failure)."""
    ctx = mp.get_context("spawn")
    q, done = ctx.Queue(), ctx.Event()
    port = _free_port()
    cons = ctx.Process(target=_consumer, args=(port, q, done))
    prod = ctx.Process(target=_producer, args=(port, q, done))
    cons.start()
    time.sleep(0.5)
    prod.start()
    res = {}
    try:
        for _ in range(2):
            role, out = q.get(timeout=timeout_s)
            res[role] = out
            if role == "consumer":
                done.set()
    except Exception as e:  # noqa: BLE001 - a child that never reported
        res.setdefault("consumer", {"error": f"no report: {type(e).__name__}"})
    finally:
        done.set()
        for p in (prod, cons):
            p.join(30)
            if p.is_alive():
                p.kill()
    p_, c_ = res.get("producer", {}), res.get("consumer", {})
    report = {"metric": "config0 CPU compression round trip + 2-process gloo PD transfer",
              "shape": [LAYERS, 2, TOKENS, HEADS, DIM], "dtype": "bf16", "seed": 0,
              "profile": "hadamard128 + minmax K4 per-channel / V4 per-token (split by head) + bitpack4",
              "error": p_.get("error") or c_.get("error")}
    if not report["error"]:
        report.update(compression_ratio=round(p_["original_bytes"] / p_["compressed_bytes"], 4),
                      wire_ratio=round(p_["original_bytes"] / p_["wire_bytes"], 4),
                      mse=round(c_["mse"], 6), mse_keys=round(c_["mse_keys"], 6),
                      mse_values=round(c_["mse_values"], 6), relative_error=round(c_["relative_error"], 5),
                      signal_power=round(c_["signal_power"], 4), compress_ms=round(p_["compress_ms"], 2),
                      send_ms=round(p_["send_ms"], 2), decompress_ms=round(c_["decompress_ms"], 2),
                      transferred=bool(p_["sent"]))
    return report


def main() -> None:
    print(json.dumps(run()))


if __name__ == "__main__":
    main()
