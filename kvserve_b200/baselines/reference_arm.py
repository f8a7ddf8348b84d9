"""The reference arm of ``bench.py``: the unmodified reference (``kvserve_v1``,
installed in ``baseline/_ref``) driven through its own public API on the same
workload as this framework's arm.

Public API used, exactly as the reference documents and tests it
(examples/external_connector_config.py:21-50, tests/test_pd_with_compression.py:399-478):
two vLLM V1 engines, a ``kv_producer`` (prefill) and a ``kv_consumer``
(decode), each built with ``KVTransferConfig(kv_connector="CompressedKVConnector",
kv_connector_module_path="kvserve_v1.connector.compressed_kv_connector", ...)``
and ``kv_connector_extra_config={"compression": <profile>}``; requests carry a
shared ``transfer_id`` in ``SamplingParams.extra_args["kv_transfer_params"]``.
KV moves through the reference's ``NcclTransport`` (ZMQ control + NCCL data)
after its modular compression pipeline.

Workload: a Llama-3.1-8B-shaped model (config.json written to a temp dir;
``load_format="dummy"`` gives random-init bf16 weights, as in this
framework's arm), random prompt token ids of the bench length, greedy
decoding with ``ignore_eos`` for the bench's output length, and the K4/V2
profile expressed in the reference's config language: ``max_value`` 16 for
keys and 4 for values on every head (``hybrid_ratio`` 0, keys per channel,
values per token, split by head), codec ``bitpack``.  The reference packs the
whole symbol buffer with one width, so values travel at 4 bits as well
(kvserve_v1/compression/compression_manager.py:300-340); ``--profile raw``
runs the reference without compression (``compression=None``).

Topology under ``torchrun`` with N ranks (N even): rank 0 drives the producer
engine on GPUs [0, N/2) (TP N/2) and rank N/2 the consumer engine on GPUs
[N/2, N); the other ranks only take part in the host barriers.  N = 1 is not
available: the reference's transport is NCCL between two engines, and NCCL
refuses two ranks on one device.

Timing (host clock; vLLM's internals are not instrumented so that the stock
path runs unmodified): every request starts after a barrier of all ranks at a
shared wall-clock instant ``t0``; the producer serves the prompt with one
output token (the KV is compressed and sent by the connector's
``wait_for_save``); the consumer, sequenced after the producer like the
reference's own PD test and vLLM's disaggregation proxy, serves the same
``transfer_id`` with the full output length.  TTFT = the consumer's first
token time - ``t0`` (vLLM's per-request ``arrival_time + first_token_latency``),
which is the maximum over ranks by construction.
"""
from __future__ import annotations

import json
import os
import socket
import statistics
import sys
import tempfile
import time
from typing import Optional

REF_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                       "baseline", "_ref")

_TORCHRUN_ENV = ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "GROUP_RANK", "GROUP_WORLD_SIZE",
                 "ROLE_RANK", "ROLE_WORLD_SIZE", "ROLE_NAME", "MASTER_ADDR", "MASTER_PORT",
                 "TORCHELASTIC_RUN_ID", "TORCHELASTIC_USE_AGENT_STORE", "TORCHELASTIC_RESTART_COUNT",
                 "TORCHELASTIC_MAX_RESTARTS", "TORCHELASTIC_ERROR_FILE", "TORCH_NCCL_ASYNC_ERROR_HANDLING",
                 "OMP_NUM_THREADS")

# Llama-3.1-8B shape with plain RoPE (theta 500000), the same architecture
# this framework's arm builds.
LLAMA_8B_CONFIG = {
    "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 4096,
    "intermediate_size": 14336, "num_attention_heads": 32, "num_key_value_heads": 8, "head_dim": 128,
    "num_hidden_layers": 32, "vocab_size": 128256, "max_position_embeddings": 131072,
    "rope_theta": 500000.0, "rms_norm_eps": 1e-5, "hidden_act": "silu", "tie_word_embeddings": False,
    "torch_dtype": "bfloat16", "bos_token_id": 128000, "eos_token_id": 128001, "attention_bias": False,
    "mlp_bias": False,
}

# The reference's compression path reads the stacked KV as [L, 2, blocks,
# block_size, H, D] (FlashAttention layout, kvserve_v1/utils/kv_utils.py:66 and
# compression/compression_manager.py:146-153); vLLM's default backend on
# B200 (FlashInfer) stores [blocks, 2, ...], which makes the consumer's
# decompress fail with a shape error.  The arm therefore selects vLLM's
# FLASH_ATTN backend, the layout the reference was validated with.
REF_ATTENTION_BACKEND = "FLASH_ATTN"

K4V2_PROFILE = {
    "enabled": True,
    "pipeline": ["quantizer", "codec"],
    "quantizer_config": {
        "model_name": "Llama-3.1-8B-Instruct", "hybrid_ratio": 0.0,
        "high_key_max_value": 16, "high_value_max_value": 4, "low_key_max_value": 16, "low_value_max_value": 4,
        "axis_key": "channel", "axis_value": "token", "split_type": "head",
    },
    "codec_config": {"codec_type": "bitpack", "bitpack_bits": 4},
    "min_compress_size": 0,
}


def unavailable_reason(world_size: int = 1) -> Optional[str]:
    """Why the arm can not run with ``world_size`` ranks here (None: it can)."""
    if not os.path.isdir(os.path.join(REF_DIR, "kvserve_v1")):
        return "reference not installed in baseline/_ref (pip install --target baseline/_ref failed)"
    if world_size < 2 or world_size % 2:
        return ("the reference's PD path is two vLLM engines joined by NCCL; it needs an even number of GPUs "
                ">= 2 (NCCL refuses two ranks on one device), so 1 GPU has no reference number")
    try:
        import vllm  # noqa: F401
    except Exception as exc:  # pragma: no cover - environment dependent
        return f"vLLM not importable: {exc!r}"
    return None


def reference_profile(name: str):
    if name == "raw":
        return None
    if name == "k4v2":
        return json.loads(json.dumps(K4V2_PROFILE))
    if os.path.exists(name):
        with open(name) as f:
            return json.load(f)
    raise SystemExit(f"unknown profile {name!r}")


def write_model_dir(cfg: dict) -> str:
    d = tempfile.mkdtemp(prefix="kvs_ref_model_")
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    return d


def _free_port_block(n: int) -> int:
    for base in range(31000, 60000, 97):
        socks = []
        try:
            for i in range(n):
                s = socket.socket()
                s.bind(("127.0.0.1", base + i))
                socks.append(s)
            return base
        except OSError:
            continue
        finally:
            for s in socks:
                s.close()
    raise RuntimeError("no free port block")


class _Barrier:
    """Host barrier over the torchrun agent's TCP store (no process group in
    this process, so vLLM's own distributed setup is untouched)."""

    def __init__(self, addr: str, port: int, rank: int, world: int, timeout_s: float = 1800.0):
        import datetime
        import torch.distributed as dist
        base = dist.TCPStore(addr, port, is_master=False, wait_for_workers=False,
                             timeout=datetime.timedelta(seconds=timeout_s))
        self.store = dist.PrefixStore("kvs_reference_arm", base)
        self.rank, self.world, self.n = rank, world, 0

    def wait(self) -> None:
        self.n += 1
        key = f"barrier{self.n}"
        self.store.add(key, 1)
        self.store.wait([f"{key}_open"]) if self.rank else self._open(key)

    def _open(self, key: str) -> None:
        while int(self.store.add(key, 0)) < self.world:
            time.sleep(0.002)
        self.store.set(f"{key}_open", "1")

    def set(self, key: str, value: str) -> None:
        self.store.set(key, value)

    def get(self, key: str) -> str:
        self.store.wait([key])
        return self.store.get(key).decode()


def run(args, emit) -> None:
    """Entry point of ``bench.py --impl reference``; rank 0 prints one JSON line."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    why = unavailable_reason(world)
    if why is not None:
        if rank == 0:
            emit({"impl": "reference", "unavailable": why})
        return
    addr, port = os.environ.get("MASTER_ADDR", "127.0.0.1"), int(os.environ["MASTER_PORT"])
    bar = _Barrier(addr, port, rank, world)
    tp = world // 2
    role = "producer" if rank == 0 else "consumer" if rank == tp else "idle"
    if rank == 0:
        bar.set("kv_port", str(_free_port_block(tp)))
    kv_port = int(bar.get("kv_port"))

    for k in _TORCHRUN_ENV:
        os.environ.pop(k, None)
    if role != "idle":
        gpus = range(0, tp) if role == "producer" else range(tp, world)
        os.environ["CUDA_VISIBLE_DEVICES"] = ",".join(str(g) for g in gpus)
        os.environ["PYTHONPATH"] = REF_DIR + os.pathsep + os.environ.get("PYTHONPATH", "")
        if REF_DIR not in sys.path:
            sys.path.insert(0, REF_DIR)

    if getattr(args, "ref_engine", "handoff") == "handoff":
        _run_handoff(args, emit, bar, rank, world, role, kv_port)
        return
    n_req = args.warmup + args.steps
    results: list[dict] = []
    llm = None
    try:
        if role != "idle":
            llm = _build_engine(args, role, tp, kv_port)
        bar.wait()  # both engines up
        import random
        rng = random.Random(1234)
        prompts = [[rng.randrange(LLAMA_8B_CONFIG["vocab_size"]) for _ in range(args.prompt_len)]
                   for _ in range(n_req)]
        sampler = None
        for i in range(n_req):
            if i == args.warmup and rank == 0:
                from ..utils.clocks import ClockSampler
                sampler = ClockSampler(list(range(world)))
                sampler.start()
            bar.wait()
            t0 = time.time()
            if rank == 0:
                bar.set(f"t0_{i}", repr(t0))
            tid = f"kvs-bench-{i}"
            if role == "producer":
                out = _generate(llm, prompts[i], 1, tid)
                bar.set(f"prefill_done_{i}", repr(time.time()))
                results.append({"prefill_ms": 1e3 * (time.time() - t0), "tokens": len(out)})
            elif role == "consumer":
                t0 = float(bar.get(f"t0_{i}"))
                p_done = float(bar.get(f"prefill_done_{i}"))
                t_start = time.time()
                o = _generate(llm, prompts[i], args.max_new, tid, want_output=True)
                t_end = time.time()
                m = o.metrics
                first = (m.arrival_time + m.first_token_latency) if m is not None and m.first_token_latency else None
                results.append({
                    "ttft_ms": 1e3 * (first - t0) if first else float("nan"),
                    "request_ms": 1e3 * (t_end - t0),
                    "prefill_ms": 1e3 * (p_done - t0),
                    "consumer_start_ms": 1e3 * (t_start - t0),
                    "tokens": len(o.outputs[0].token_ids),
                })
                bar.set(f"consumer_{i}", json.dumps(results[-1]))
        bar.wait()
        clocks = sampler.stop() if sampler else None
        if rank == 0:
            rows = [json.loads(bar.get(f"consumer_{i}")) for i in range(args.warmup, n_req)]
            ttft = [r["ttft_ms"] for r in rows]
            req = [r["request_ms"] for r in rows]
            pre = [r["prefill_ms"] for r in rows]
            emit({
                "impl": "reference",
                "metric": args.metric,
                "value": round(statistics.median(ttft), 3),
                "unit": "ms (TTFT p50)",
                "n_gpus": world,
                "steps": args.steps,
                "warmup": args.warmup,
                "ms_per_step": round(statistics.mean(req), 3),
                "higher_is_better": False,
                "scaling": "strong",
                "vs_baseline": None,
                "dtype": "bf16",
                "data": "synthetic (vLLM dummy random-init weights of the named architecture, uniform-random "
                        "prompt token ids)",
                "prefill_ms_p50": round(statistics.median(pre), 3),
                "handoff_to_first_token_ms_p50": round(statistics.median(t - p for t, p in zip(ttft, pre)), 3),
                "decode_ms_per_token": round(statistics.median(r - t for r, t in zip(req, ttft))
                                             / max(1, args.max_new - 1), 4),
                "output_tokens": rows[0]["tokens"],
                "config": {"model": "llama-3.1-8b", "layers": LLAMA_8B_CONFIG["num_hidden_layers"],
                           "global_batch": 1, "seq_len": args.prompt_len, "max_new_tokens": args.max_new,
                           "parallelism": f"{tp}P{tp}D-tp{tp}", "profile": args.profile,
                           "engine": f"vLLM V1 + kvserve_v1 CompressedKVConnector/NcclTransport "
                                     f"(attention {REF_ATTENTION_BACKEND}, "
                                     f"enforce_eager={not getattr(args, 'ref_cuda_graphs', False)}, "
                                     f"chunked prefill off)",
                           "l2": "inputs larger than L2 (16 GB weights, 1 GiB raw KV per request)"},
                "e2e": {"value": round(statistics.median(ttft), 3),
                        "unit": "ms (TTFT p50, host clock from the shared request start to the consumer's first "
                                "token through vLLM's public LLM.generate API)",
                        "h2d_bytes_per_step": 8 * args.prompt_len, "d2h_bytes_per_step": 8 * (args.max_new + 1),
                        "request_ms_p50": round(statistics.median(req), 3)},
                "timing": "host clock (the reference's stock path is not instrumented with device events)",
                "gpu_launches": None,
                "clocks": clocks,
            })
    finally:
        if llm is not None:
            _shutdown(llm)


VLLM_INCOMPATIBLE = ("kvserve_v1's CompressedKVConnector does not run on the image's vLLM 0.22: its consumer "
                     "injects KV with forward_context.virtual_engine (removed; layer.kv_cache is one tensor), "
                     "so the decode engine dies on the first request; TTFT of the reference is unmeasured, "
                     "its KV hand-off path is measured instead (kv_transfer_ms_p50)")


def _run_handoff(args, emit, bar, rank: int, world: int, role: str, kv_port: int) -> None:
    """The reference's KV hand-off data path exactly as its connector runs it
    (compressed_kv_connector.py:393-470 producer, 235-372 consumer), without
    vLLM: ``KVCompressionAdapter.compress`` of the stacked request KV
    ``[L, 2, blocks, block_size, H, D]``, ``build_wire``, ``NcclTransport
    .send_bundle``; on the consumer ``drain_received``, ``restore_from_wire``,
    ``decompress`` and ``inject_kv_into_layer_by_blocks`` into a paged cache.
    Time = consumer's KV-in-cache instant - shared start (host clock after
    device synchronisation), i.e. the per-request KV-transfer time, max over
    ranks by construction.  Synthetic N(0, 1) KV of the bench shape."""
    import torch
    L, H, D, bs = LLAMA_8B_CONFIG["num_hidden_layers"], LLAMA_8B_CONFIG["num_key_value_heads"], 128, 16
    nblk = (args.prompt_len - 1 + bs - 1) // bs
    n_req = args.warmup + args.steps
    profile = reference_profile(args.profile)
    rows = []
    t = None
    if role != "idle":
        torch.cuda.set_device(0)
        from kvserve_v1.transport.nccl_transport import NcclTransport
        from kvserve_v1.compression.manager import KVCompressionAdapter, add_sentinel
        t = NcclTransport(is_sender=(role == "producer"), host="127.0.0.1", port=kv_port, local_rank=0,
                          channel_rank=0, recv_buffer_size=4 * 2 ** 30)
        ad = KVCompressionAdapter(profile, H, D) if profile is not None else None
        names = [f"model.layers.{i}.self_attn.attn" for i in range(L)]
        g = torch.Generator(device="cuda").manual_seed(1234)
        if role == "producer":
            from kvserve_v1.compression.wire import build_wire
            from kvserve_v1.connector.compressed_kv_connector import _max_nccl_chunk_bytes
            stacked = torch.randn((L, 2, nblk, bs, H, D), generator=g, device="cuda").to(torch.bfloat16)
        else:
            from kvserve_v1.compression.wire import CompressedWire, restore_from_wire
            from kvserve_v1.compression.manager import strip_sentinel, is_compressed_layer_names
            from kvserve_v1.utils.kv_utils import inject_kv_into_layer_by_blocks
            cache = torch.empty((L, 2, nblk + 64, bs, H, D), dtype=torch.bfloat16, device="cuda")
            block_ids = list(range(7, 7 + nblk))
    sampler = None
    try:
        for i in range(n_req):
            if i == args.warmup and rank == 0:
                from ..utils.clocks import ClockSampler
                sampler = ClockSampler(list(range(world)))
                sampler.start()
            if t is not None:
                torch.cuda.synchronize()
            bar.wait()
            if rank == 0:
                bar.set(f"t0_{i}", repr(time.time()))
            tid = f"kvs-ref-{i}"
            if role == "producer":
                t0 = float(bar.get(f"t0_{i}"))
                if ad is not None:
                    c = ad.compress(stacked, tid)
                    wire = build_wire(c, _max_nccl_chunk_bytes())
                    t.send_bundle(tid, add_sentinel(names), wire.meta, wire.body_chunks, wire.aux_tensors)
                    nbytes = wire.nbytes
                else:
                    t.send(tid, names, stacked)
                    nbytes = stacked.numel() * 2
                t.wait_for_sent()
                torch.cuda.synchronize()
                bar.set(f"sent_{i}", json.dumps({"sent_ms": 1e3 * (time.time() - t0), "bytes": int(nbytes)}))
            elif role == "consumer":
                t0 = float(bar.get(f"t0_{i}"))
                t.set_expected_requests([tid])
                got = None
                deadline = time.monotonic() + 300
                while got is None and time.monotonic() < deadline:
                    for key, payloads in t.drain_received().items():
                        if key == tid:
                            got = payloads[0]
                    if got is None:
                        time.sleep(0.001)
                if got is None:
                    raise RuntimeError(f"reference transport timed out on {tid}")
                layer_names, payload = got
                nb = t.payload_nbytes(payload)
                if is_compressed_layer_names(layer_names):
                    wire = CompressedWire(meta=payload["meta"], body_chunks=payload["body_chunks"],
                                          aux_tensors=payload["aux_tensors"])
                    kv = ad.decompress(restore_from_wire(wire))
                else:
                    kv = payload
                for li in range(L):
                    inject_kv_into_layer_by_blocks(cache[li], kv[li], block_ids, tid)
                torch.cuda.synchronize()
                t.release_received(tid, nb)
                bar.set(f"done_{i}", repr(1e3 * (time.time() - t0)))
        bar.wait()
        clocks = sampler.stop() if sampler else None
        if rank == 0:
            tm = [float(bar.get(f"done_{i}")) for i in range(args.warmup, n_req)]
            sent = [json.loads(bar.get(f"sent_{i}")) for i in range(args.warmup, n_req)]
            raw = 2 * L * nblk * bs * H * D * 2
            emit({
                "impl": "reference",
                "unavailable": VLLM_INCOMPATIBLE,
                "metric": args.metric,
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "kv_transfer_ms_p50": round(statistics.median(tm), 3),
                "kv_send_ms_p50": round(statistics.median(x["sent_ms"] for x in sent), 3),
                "kv_payload_bytes_per_request": sent[0]["bytes"],
                "kv_raw_bytes_per_request": raw,
                "compression_ratio": round(raw / sent[0]["bytes"], 3),
                "config": {"model": "llama-3.1-8b (KV shape only)", "layers": L, "seq_len": args.prompt_len,
                           "profile": args.profile, "path": "kvserve_v1 KVCompressionAdapter + CompressedWire + "
                                                           "NcclTransport, 1 producer -> 1 consumer",
                           "data": "synthetic N(0,1) bf16 KV"},
                "timing": "host clock after device synchronisation, consumer end - shared start",
                "clocks": clocks,
            })
    finally:
        if t is not None:
            for m in ("shutdown", "close"):
                fn = getattr(t, m, None)
                if callable(fn):
                    try:
                        fn()
                    except Exception:
                        pass
                    break


def _build_engine(args, role: str, tp: int, kv_port: int):
    from vllm import LLM
    from vllm.config import KVTransferConfig
    model_dir = write_model_dir(LLAMA_8B_CONFIG)
    kv_cfg = KVTransferConfig(
        kv_connector="CompressedKVConnector",
        kv_connector_module_path="kvserve_v1.connector.compressed_kv_connector",
        kv_role="kv_producer" if role == "producer" else "kv_consumer",
        kv_rank=0 if role == "producer" else 1,
        kv_parallel_size=2,
        kv_ip="127.0.0.1",
        kv_port=kv_port,
        kv_connector_extra_config={"compression": reference_profile(args.profile)},
    )
    max_len = args.prompt_len + args.max_new
    return LLM(model=model_dir, load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16",
               tensor_parallel_size=tp, max_model_len=max_len, max_num_batched_tokens=max_len,
               enable_chunked_prefill=False, enable_prefix_caching=False, gpu_memory_utilization=0.6,
               enforce_eager=not getattr(args, "ref_cuda_graphs", False), kv_transfer_config=kv_cfg,
               disable_log_stats=False, seed=0, attention_backend=REF_ATTENTION_BACKEND)


def _generate(llm, prompt: list[int], max_tokens: int, transfer_id: str, want_output: bool = False):
    from vllm import SamplingParams
    from vllm.inputs import TokensPrompt
    sp = SamplingParams(max_tokens=max_tokens, temperature=0.0, ignore_eos=True, detokenize=False,
                        extra_args={"kv_transfer_params": {"transfer_id": transfer_id}})
    outs = llm.generate([TokensPrompt(prompt_token_ids=prompt)], sampling_params=sp, use_tqdm=False)
    return outs[0] if want_output else outs[0].outputs[0].token_ids


def _shutdown(llm) -> None:
    core = getattr(getattr(llm, "llm_engine", None), "engine_core", None)
    stop = getattr(core, "shutdown", None)
    if callable(stop):
        try:
            stop()
        except Exception:
            pass
