"""The reference arm of ``bench.py``: the reference (``kvserve_v1``, installed
unmodified in ``baseline/_ref``) driven through its own public API on the
same workload as this framework's arm.

Public API used, as the reference documents and tests it
(examples/external_connector_config.py:21-50, tests/test_pd_with_compression.py:399-478,
tests/test_kvserve.py:411-614): two vLLM V1 engines, a ``kv_producer``
(prefill) and a ``kv_consumer`` (decode), each built with
``KVTransferConfig(kv_connector="CompressedKVConnector",
kv_connector_module_path="kvserve_v1.connector.compressed_kv_connector", ...)``
and ``kv_connector_extra_config={"compression": <profile>}``; requests carry a
shared ``transfer_id`` in ``SamplingParams.extra_args["kv_transfer_params"]``.
KV moves through the reference's ``NcclTransport`` (ZMQ control + NCCL data)
after its modular compression pipeline.

The run has three parts, all on reference code:

1. **Stock check** (tiny model, one request): the unmodified stack on the
   image's vLLM 0.22.  Its consumer fails in ``start_load_kv``: it reads
   ``forward_context.virtual_engine`` and indexes ``layer.kv_cache`` by it,
   an API of the older vLLM it was written for.  The captured exception is
   printed in the JSON line (``stock_path``).
2. **PD serving** (the metric): the same engines with a vLLM-API adapter
   (:mod:`kvserve_b200.baselines.vllm_compat`, a vLLM plugin that hands the
   connector the forward context in the older shape; the reference's code is
   not changed).  TTFT per request, host clock.
3. **Hand-off alone**: the reference connector's data path without vLLM
   (compress, wire, ``NcclTransport``, decompress, inject) on synthetic KV of
   the request's shape: the per-request KV-transfer time.

Plus the reconstruction error of the profile on the synthetic KV that the
framework's arm measures too.

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
[N/2, N); the other ranks only take part in the host barriers.  N = 1 cannot
run the pair (the reference's transport is NCCL between two engines, and NCCL
refuses two ranks on one device); it reports the labelled composite of
:func:`run_single_gpu` instead.

Timing (host clock; vLLM's internals are not instrumented so that the stock
path runs as shipped): every request starts after a barrier of all ranks at a
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

REPO_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
REF_DIR = os.path.join(REPO_ROOT, "baseline", "_ref")

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


NCCL_ONE_GPU = ("the reference's PD path is two vLLM engines joined by NCCL, which refuses two ranks on one "
                "device")


def unavailable_reason(world_size: int = 1) -> Optional[str]:
    """Why the arm can not run with ``world_size`` ranks here (None: it can;
    one GPU runs the composite of :func:`run_single_gpu`)."""
    if not os.path.isdir(os.path.join(REF_DIR, "kvserve_v1")):
        return "reference not installed in baseline/_ref (pip install --target baseline/_ref failed)"
    if world_size > 1 and world_size % 2:
        return f"{NCCL_ONE_GPU}; it needs an even number of GPUs"
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


def _free_port_block(n: int, first: int = 31000) -> int:
    for base in range(first, 60000, 97):
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

    def wait(self, name: Optional[str] = None, allow_failed: bool = False) -> None:
        """Barrier of all ranks.  Unnamed barriers are numbered in call order;
        while one is pending, a published failure ends it with ArmFailure
        (unless ``allow_failed``: the barrier that every rank reaches on every
        path is named and waits regardless)."""
        if name is None:
            self.n += 1
            name = f"barrier{self.n}"
        self.store.add(name, 1)
        while True:
            if self.rank == 0 and int(self.store.add(name, 0)) >= self.world:
                self.store.set(f"{name}_open", "1")
            if self.store.check([f"{name}_open"]):
                return
            if not allow_failed and self.failed():
                raise ArmFailure(self.failed())
            time.sleep(0.002)

    def failed(self) -> Optional[str]:
        if self.store.check(["failed"]):
            return self.store.get("failed").decode()
        return None

    def set(self, key: str, value: str) -> None:
        self.store.set(key, value)

    def get(self, key: str) -> str:
        while not self.store.check([key]):
            if self.failed() and key != "failed":
                raise ArmFailure(self.failed())
            time.sleep(0.002)
        return self.store.get(key).decode()


class ArmFailure(RuntimeError):
    """A role of the reference arm failed; the message is the captured error."""


def _ref_env(role: str, tp: int, world: int, adapter_dir: Optional[str]) -> None:
    """Environment of a reference role: its GPUs, the reference package and,
    for the adapted run, the vLLM plugin directory on the import path."""
    gpus = range(0, tp) if role == "producer" else range(tp, world)
    os.environ["CUDA_VISIBLE_DEVICES"] = ",".join(str(g) for g in gpus)
    paths = [REF_DIR, REPO_ROOT] + ([adapter_dir] if adapter_dir else [])
    os.environ["PYTHONPATH"] = os.pathsep.join(paths + [os.environ.get("PYTHONPATH", "")]).rstrip(os.pathsep)
    for pth in reversed(paths):
        if pth not in sys.path:
            sys.path.insert(0, pth)


def _role_call(bar: "_Barrier", key: str, fn):
    """Run ``fn`` and publish failure (``failed`` key) so no rank waits forever."""
    try:
        return fn()
    except BaseException as exc:  # noqa: BLE001 - the text is the result
        msg = f"{key}: {type(exc).__name__}: {exc}"[:600]
        bar.set("failed", msg)
        raise ArmFailure(msg) from exc


def run(args, emit) -> None:
    """Entry point of ``bench.py --impl reference``; rank 0 prints one JSON line."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    why = unavailable_reason(world)
    if why is not None:
        if rank == 0:
            emit({"impl": "reference", "unavailable": why})
        return
    if world == 1:
        if getattr(args, "ref_engine", "vllm") != "vllm":
            emit({"impl": "reference", "unavailable": NCCL_ONE_GPU})
            return
        emit(run_single_gpu(args))
        return
    addr, port = os.environ.get("MASTER_ADDR", "127.0.0.1"), int(os.environ["MASTER_PORT"])
    bar = _Barrier(addr, port, rank, world)
    tp = world // 2
    role = "producer" if rank == 0 else "consumer" if rank == tp else "idle"
    if rank == 0:
        bar.set("ports", json.dumps([_free_port_block(max(2, tp), 31000 + 200 * i) for i in range(3)]))
    ports = json.loads(bar.get("ports"))
    for k in _TORCHRUN_ENV:
        os.environ.pop(k, None)
    mode = getattr(args, "ref_engine", "vllm")
    out: dict = {"impl": "reference", "metric": args.metric, "n_gpus": world, "steps": args.steps,
                 "warmup": args.warmup}
    try:
        if mode == "handoff":
            if role != "idle":
                _ref_env(role, tp, world, None)
            out.update(_run_handoff(args, bar, rank, world, role, ports[2]))
            out["unavailable"] = "hand-off only (--ref-engine handoff): no TTFT"
        else:
            stock = _stock_check(args, bar, rank, role, tp, world, ports[0])
            out["stock_path"] = stock
            if mode == "stock":
                out["unavailable"] = f"stock reference on vLLM 0.22: {stock}"
            else:
                adapter_dir = None
                if role != "idle":
                    from .vllm_compat import install_entry_point
                    adapter_dir = install_entry_point(tempfile.mkdtemp(prefix="kvs_ref_vllm_plugin_"))
                    _ref_env(role, tp, world, adapter_dir)
                out.update(_run_vllm(args, bar, rank, world, role, tp, ports[1]))
                bar.wait()
                ho = _run_handoff(args, bar, rank, world, role, ports[2])
                if rank == 0:
                    out["kv_transfer_ms_p50"] = ho.pop("kv_transfer_ms_p50")
                    out["kv_transfer"] = ho
                    out["recon"] = _reference_recon(args)
    except ArmFailure as exc:
        out = {"impl": "reference", "unavailable": str(exc), "stock_path": out.get("stock_path")}
    bar.wait("final", allow_failed=True)
    if rank == 0:
        if bar.failed():
            out = {"impl": "reference", "unavailable": f"reference run failed: {bar.failed()}",
                   "stock_path": out.get("stock_path")}
        emit(out)


def _local_handoff(args, n_req: int) -> dict:
    """The reference connector's data path for one request's KV on one GPU:
    ``compress`` of the stacked ``[L, 2, blocks, block_size, H, D]`` KV,
    ``build_wire``, the payload tensors copied as the transport would land
    them, ``restore_from_wire``, ``decompress`` and
    ``inject_kv_into_layer_by_blocks`` into a paged cache (all 8 KV heads,
    TP 1).  Host clock after device synchronisation; the median."""
    import torch
    from kvserve_v1.compression.manager import KVCompressionAdapter
    from kvserve_v1.compression.wire import CompressedWire, build_wire, restore_from_wire
    from kvserve_v1.connector.compressed_kv_connector import _max_nccl_chunk_bytes
    from kvserve_v1.utils.kv_utils import inject_kv_into_layer_by_blocks
    L, H, D, bs = LLAMA_8B_CONFIG["num_hidden_layers"], LLAMA_8B_CONFIG["num_key_value_heads"], 128, 16
    nblk = (args.prompt_len - 1 + bs - 1) // bs
    profile = reference_profile(args.profile)
    g = torch.Generator(device="cuda").manual_seed(1234)
    stacked = torch.randn((L, 2, nblk, bs, H, D), generator=g, device="cuda").to(torch.bfloat16)
    cache = torch.empty((L, 2, nblk + 64, bs, H, D), dtype=torch.bfloat16, device="cuda")
    block_ids = list(range(7, 7 + nblk))
    ad = KVCompressionAdapter(profile, H, D) if profile is not None else None
    times, nbytes = [], stacked.numel() * 2
    for i in range(n_req):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        if ad is not None:
            c = ad.compress(stacked, f"kvs-ref-local-{i}")
            w = build_wire(c, _max_nccl_chunk_bytes())
            landed = CompressedWire(meta=w.meta, body_chunks=[b.clone() for b in w.body_chunks],
                                    aux_tensors=[a.clone() for a in w.aux_tensors])
            kv = ad.decompress(restore_from_wire(landed))
            nbytes = w.nbytes
        else:
            kv = stacked.clone()
        for li in range(L):
            inject_kv_into_layer_by_blocks(cache[li], kv[li], block_ids, f"kvs-ref-local-{i}")
        torch.cuda.synchronize()
        times.append(1e3 * (time.perf_counter() - t0))
    del stacked, cache
    torch.cuda.empty_cache()
    kept = times[args.warmup:] or times
    return {"handoff_ms_p50": round(statistics.median(kept), 3), "payload_bytes": int(nbytes),
            "raw_bytes": 2 * L * nblk * bs * H * D * 2}


def run_single_gpu(args) -> dict:
    """One GPU: the reference cannot run its PD pair here (its transport is
    an NCCL communicator between two engines).  The arm reports a composite
    built only from reference code on the same request: the TTFT of vLLM (the
    reference's engine) prefilling the prompt on this GPU, plus the
    reference connector's KV data path for that request without the network
    (:func:`_local_handoff`), plus one decode step (the decode engine
    recomputes the last prompt token before it samples).  Labelled
    ``composite``; a failure prints ``unavailable`` with its reason."""
    out = {"impl": "reference", "metric": args.metric, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup}
    import torch
    if not torch.cuda.is_available():
        return {"impl": "reference", "unavailable": f"{NCCL_ONE_GPU}; no GPU visible for the one-GPU composite"}
    llm = None
    try:
        os.environ["CUDA_VISIBLE_DEVICES"] = os.environ.get("CUDA_VISIBLE_DEVICES", "0")
        for pth in (REF_DIR, REPO_ROOT):
            if pth not in sys.path:
                sys.path.insert(0, pth)
        from vllm import LLM
        n_req = args.warmup + args.steps
        max_len = args.prompt_len + args.max_new
        llm = LLM(model=write_model_dir(LLAMA_8B_CONFIG), load_format="dummy", skip_tokenizer_init=True,
                  dtype="bfloat16", max_model_len=max_len, max_num_batched_tokens=max_len,
                  enable_chunked_prefill=False, enable_prefix_caching=False, gpu_memory_utilization=0.6,
                  enforce_eager=not getattr(args, "ref_cuda_graphs", False), disable_log_stats=False, seed=0,
                  attention_backend=REF_ATTENTION_BACKEND)
        import random
        rng = random.Random(1234)
        ttft, step = [], []
        for i in range(n_req):
            prompt = [rng.randrange(LLAMA_8B_CONFIG["vocab_size"]) for _ in range(args.prompt_len)]
            t0 = time.time()
            o = _generate(llm, prompt, 2, f"kvs-ref-1gpu-{i}", want_output=True)
            t1 = time.time()
            m = o.metrics
            first = (m.arrival_time + m.first_token_latency) if m is not None and m.first_token_latency else None
            if first is None:
                raise RuntimeError("vLLM reported no first-token time")
            if i >= args.warmup:
                ttft.append(1e3 * (first - t0))
                step.append(1e3 * (t1 - first))
        _shutdown(llm)
        llm = None
        import gc
        gc.collect()
        ho = _local_handoff(args, n_req)
        prefill, dstep = statistics.median(ttft), statistics.median(step)
        value = prefill + ho["handoff_ms_p50"] + dstep
        out.update({
            "value": round(value, 3), "unit": "ms (TTFT p50, composite)", "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "composite": True, "same_config": True,
            "composite_parts": {"vllm_prefill_ttft_ms_p50": round(prefill, 3),
                                "reference_kv_data_path_ms_p50": ho["handoff_ms_p50"],
                                "decode_step_ms_p50": round(dstep, 3)},
            "kv_transfer_ms_p50": ho["handoff_ms_p50"],
            "compression_ratio": round(ho["raw_bytes"] / ho["payload_bytes"], 3),
            "data": "synthetic (vLLM dummy random-init weights of the named architecture, uniform-random prompt "
                    "token ids; N(0,1) KV for the data path)",
            "config": {"model": "llama-3.1-8b", "layers": LLAMA_8B_CONFIG["num_hidden_layers"], "global_batch": 1,
                       "seq_len": args.prompt_len, "max_new_tokens": args.max_new,
                       "parallelism": "colocated-1gpu (composite of reference parts)", "profile": args.profile,
                       "engine": f"vLLM 0.22 V1 (attention {REF_ATTENTION_BACKEND}) + kvserve_v1 connector data "
                                 f"path (KVCompressionAdapter, CompressedWire, kv_utils) without its NCCL transport"},
            "why_composite": NCCL_ONE_GPU,
            "timing": "host clock (vLLM first-token metrics; device-synchronised data path)",
            "gpu_launches": None,
            "recon": _reference_recon(args),
        })
        return out
    except BaseException as exc:  # noqa: BLE001 - the arm always prints one line
        return {"impl": "reference", "unavailable": f"{NCCL_ONE_GPU}; the one-GPU composite failed: "
                                                    f"{type(exc).__name__}: {str(exc)[:300]}"}
    finally:
        if llm is not None:
            _shutdown(llm)


def _tiny_model_dir() -> str:
    cfg = dict(LLAMA_8B_CONFIG, hidden_size=256, intermediate_size=512, num_attention_heads=4,
               num_key_value_heads=2, head_dim=64, num_hidden_layers=2, vocab_size=1024,
               max_position_embeddings=4096)
    return write_model_dir(cfg)


def _stock_child(role: str, kv_port: int, q) -> None:
    """One role of the stock check in a child process: a tiny model, the
    unmodified reference connector, vLLM in-process (so an exception raised
    in the connector reaches ``generate`` with its own text)."""
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
    try:
        from vllm import LLM, SamplingParams
        from vllm.config import KVTransferConfig
        from vllm.inputs import TokensPrompt
        kv_cfg = KVTransferConfig(kv_connector="CompressedKVConnector",
                                  kv_connector_module_path="kvserve_v1.connector.compressed_kv_connector",
                                  kv_role="kv_producer" if role == "producer" else "kv_consumer",
                                  kv_rank=0 if role == "producer" else 1, kv_parallel_size=2, kv_ip="127.0.0.1",
                                  kv_port=kv_port, kv_connector_extra_config={"compression": None})
        llm = LLM(model=_tiny_model_dir(), load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16",
                  max_model_len=256, enforce_eager=True, gpu_memory_utilization=0.1, kv_transfer_config=kv_cfg,
                  attention_backend=REF_ATTENTION_BACKEND, seed=0)
        q.put(("ready", ""))
        # the consumer's connector waits (its own load timeout) for the payload,
        # so both roles can issue the request as soon as their engine is up
        sp = SamplingParams(max_tokens=2, temperature=0.0, ignore_eos=True, detokenize=False,
                            extra_args={"kv_transfer_params": {"transfer_id": "kvs-stock-0"}})
        llm.generate([TokensPrompt(prompt_token_ids=list(range(1, 65)))], sampling_params=sp, use_tqdm=False)
        q.put(("ok", "served one request"))
    except BaseException as exc:  # noqa: BLE001 - reported to the parent
        import traceback
        tb = traceback.extract_tb(exc.__traceback__)
        where = next((f"{os.path.basename(f.filename)}:{f.lineno}" for f in reversed(tb)
                      if "kvserve_v1" in f.filename), "")
        q.put(("error", f"{type(exc).__name__}: {exc}" + (f" (at {where})" if where else "")))
    finally:
        # flush the queue's feeder thread before leaving without running the
        # engine's and the transport's exit handlers (their threads may block)
        q.close()
        q.join_thread()
        os._exit(0)


def _stock_check(args, bar: "_Barrier", rank: int, role: str, tp: int, world: int, kv_port: int) -> str:
    """Run one request through the unmodified stack (tiny model, TP 1) and
    return what happened on the consumer (the captured exception text)."""
    import multiprocessing as mp
    result = ""
    if role != "idle":
        _ref_env(role, tp, world, None)
        os.environ["CUDA_VISIBLE_DEVICES"] = str(0 if role == "producer" else tp)   # TP 1
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        child = ctx.Process(target=_stock_child, args=(role, kv_port, q), daemon=True)
        child.start()
        try:
            state, msg = q.get(timeout=240)
            if state == "ready":
                bar.set(f"stock_ready_{role}", "1")
                state, msg = q.get(timeout=180)
            result = msg
        except Exception as exc:  # noqa: BLE001 - a stuck child is a result too
            result = f"no answer from the {role} ({type(exc).__name__})"
        finally:
            child.join(10)
            if child.is_alive():
                child.kill()
                child.join(10)
        bar.set(f"stock_{role}", result)
    bar.wait("stock_done", allow_failed=True)
    return bar.get("stock_consumer") if rank == 0 else result


def _run_vllm(args, bar: "_Barrier", rank: int, world: int, role: str, tp: int, kv_port: int) -> dict:
    """PD serving through vLLM with the reference connector (adapted API)."""
    n_req = args.warmup + args.steps
    llm = None
    try:
        if role != "idle":
            llm = _role_call(bar, f"{role} engine start", lambda: _build_engine(args, role, tp, kv_port))
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
                _role_call(bar, "producer request", lambda: _generate(llm, prompts[i], 1, tid))
                bar.set(f"prefill_done_{i}", repr(time.time()))
            elif role == "consumer":
                t0 = float(bar.get(f"t0_{i}"))
                p_done = float(bar.get(f"prefill_done_{i}"))
                t_start = time.time()
                o = _role_call(bar, "consumer request",
                               lambda: _generate(llm, prompts[i], args.max_new, tid, want_output=True))
                t_end = time.time()
                m = o.metrics
                first = (m.arrival_time + m.first_token_latency) if m is not None and m.first_token_latency else None
                bar.set(f"consumer_{i}", json.dumps({
                    "ttft_ms": 1e3 * (first - t0) if first else float("nan"),
                    "request_ms": 1e3 * (t_end - t0), "prefill_ms": 1e3 * (p_done - t0),
                    "consumer_start_ms": 1e3 * (t_start - t0), "tokens": len(o.outputs[0].token_ids)}))
        bar.wait()
        clocks = sampler.stop() if sampler else None
    finally:
        if llm is not None:
            _shutdown(llm)
    if rank != 0:
        return {}
    rows = [json.loads(bar.get(f"consumer_{i}")) for i in range(args.warmup, n_req)]
    ttft = [r["ttft_ms"] for r in rows]
    req = [r["request_ms"] for r in rows]
    pre = [r["prefill_ms"] for r in rows]
    return {
        "value": round(statistics.median(ttft), 3),
        "unit": "ms (TTFT p50)",
        "ms_per_step": round(statistics.mean(req), 3),
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (vLLM dummy random-init weights of the named architecture, uniform-random "
                "prompt token ids)",
        "prefill_and_send_ms_p50": round(statistics.median(pre), 3),
        "handoff_to_first_token_ms_p50": round(statistics.median(t - p for t, p in zip(ttft, pre)), 3),
        "decode_ms_per_token": round(statistics.median(r - t for r, t in zip(req, ttft))
                                     / max(1, args.max_new - 1), 4),
        "output_tokens": rows[0]["tokens"],
        "config": {"model": "llama-3.1-8b", "layers": LLAMA_8B_CONFIG["num_hidden_layers"],
                   "global_batch": 1, "seq_len": args.prompt_len, "max_new_tokens": args.max_new,
                   "parallelism": f"{tp}P{tp}D-tp{tp}", "profile": args.profile,
                   "engine": f"vLLM 0.22 V1 + kvserve_v1 CompressedKVConnector/NcclTransport "
                             f"(attention {REF_ATTENTION_BACKEND}, "
                             f"enforce_eager={not getattr(args, 'ref_cuda_graphs', False)}, chunked prefill off)",
                   "vllm_api_adapter": "kvserve_b200.baselines.vllm_compat: forward_context.virtual_engine = 0 "
                                       "and layer.kv_cache as a per-virtual-engine list for the connector's "
                                       "start_load_kv (reference code unchanged)",
                   "l2": "inputs larger than L2 (16 GB weights, 1 GiB raw KV per request)"},
        "e2e": {"value": round(statistics.median(ttft), 3),
                "unit": "ms (TTFT p50, host clock from the shared request start to the consumer's first "
                        "token through vLLM's public LLM.generate API)",
                "h2d_bytes_per_step": 8 * args.prompt_len, "d2h_bytes_per_step": 8 * (args.max_new + 1),
                "request_ms_p50": round(statistics.median(req), 3)},
        "timing": "host clock (the reference's stock path is not instrumented with device events)",
        "gpu_launches": None,
        "clocks": clocks,
    }


def _reference_recon(args) -> Optional[dict]:
    """Reconstruction error and ratio of the reference's own adapter on the
    synthetic KV the framework's arm measures (same generator, 4 layers)."""
    profile = reference_profile(args.profile)
    if profile is None:
        return {"rel_mse": 0.0, "mse": 0.0, "compression_ratio": 1.0}
    import torch
    from kvserve_v1.compression.manager import KVCompressionAdapter
    from ..engine.fidelity import error_stats, synthetic_kv
    H, D, bs, L = LLAMA_8B_CONFIG["num_key_value_heads"], 128, 16, 4
    T = (args.prompt_len // bs) * bs
    kv = synthetic_kv(L, T, H, D, 0, torch.device("cuda", 0))          # [L, 2, T, H, D]
    stacked = kv.view(L, 2, T // bs, bs, H, D)
    ad = KVCompressionAdapter(profile, H, D)
    c = ad.compress(stacked, "kvs-recon")
    out = ad.decompress(c).reshape(L, 2, T, H, D)
    torch.cuda.synchronize()
    st = error_stats(kv, out)
    st.update({"compression_ratio": round(c.original_size / c.compressed_size, 3), "layers": L, "tokens": T,
               "kv_heads": H, "head_dim": D,
               "data": "synthetic: V ~ N(0,1), K ~ N(0,1) with 4 outlier channels x8 per head, seed 0"})
    return st


def _run_handoff(args, bar, rank: int, world: int, role: str, kv_port: int) -> dict:
    """The reference's KV hand-off data path exactly as its connector runs it
    (compressed_kv_connector.py:393-470 producer, 235-372 consumer), without
    vLLM: ``KVCompressionAdapter.compress`` of the stacked request KV
    ``[L, 2, blocks, block_size, H, D]``, ``build_wire``, ``NcclTransport
    .send_bundle``; on the consumer ``drain_received``, ``restore_from_wire``,
    ``decompress`` and ``inject_kv_into_layer_by_blocks`` into a paged cache.
    One channel with one TP rank's heads (``8 / TP``; the connector runs one
    such channel per TP rank, in parallel).  Time = consumer's KV-in-cache
    instant - shared start (host clock after device synchronisation), i.e.
    the per-request KV-transfer time, max over ranks by construction.
    Synthetic N(0, 1) KV of the bench shape.  Returns rank 0's summary."""
    import torch
    tp = max(1, world // 2)
    L, D, bs = LLAMA_8B_CONFIG["num_hidden_layers"], 128, 16
    H = max(1, LLAMA_8B_CONFIG["num_key_value_heads"] // tp)
    nblk = (args.prompt_len - 1 + bs - 1) // bs
    n_req = args.warmup + args.steps
    profile = reference_profile(args.profile)
    t = None
    try:
        if role != "idle":
            torch.cuda.set_device(0)
            from kvserve_v1.transport.nccl_transport import NcclTransport
            from kvserve_v1.compression.manager import KVCompressionAdapter, add_sentinel
            t = _role_call(bar, f"{role} transport", lambda: NcclTransport(
                is_sender=(role == "producer"), host="127.0.0.1", port=kv_port, local_rank=0, channel_rank=0,
                recv_buffer_size=4 * 2 ** 30))
            ad = KVCompressionAdapter(profile, H, D, tp_rank=0, tp_size=tp) if profile is not None else None
            names = [f"model.layers.{i}.self_attn.attn" for i in range(L)]
            g = torch.Generator(device="cuda").manual_seed(1234)
            if role == "producer":
                from kvserve_v1.compression.wire import build_wire
                from kvserve_v1.connector.compressed_kv_connector import _max_nccl_chunk_bytes
                stacked = torch.randn((L, 2, nblk, bs, H, D), generator=g, device="cuda").to(torch.bfloat16)
            else:
                from kvserve_v1.compression.wire import CompressedWire, restore_from_wire
                from kvserve_v1.compression.manager import is_compressed_layer_names
                from kvserve_v1.utils.kv_utils import inject_kv_into_layer_by_blocks
                cache = torch.empty((L, 2, nblk + 64, bs, H, D), dtype=torch.bfloat16, device="cuda")
                block_ids = list(range(7, 7 + nblk))
        for i in range(n_req):
            if t is not None:
                torch.cuda.synchronize()
            bar.wait()
            if rank == 0:
                bar.set(f"h_t0_{i}", repr(time.time()))
            tid = f"kvs-ref-{i}"
            if role == "producer":
                t0 = float(bar.get(f"h_t0_{i}"))

                def send():
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
                    return nbytes
                nbytes = _role_call(bar, "producer hand-off", send)
                bar.set(f"h_sent_{i}", json.dumps({"sent_ms": 1e3 * (time.time() - t0), "bytes": int(nbytes)}))
            elif role == "consumer":
                t0 = float(bar.get(f"h_t0_{i}"))

                def receive():
                    t.set_expected_requests([tid])
                    got = None
                    deadline = time.monotonic() + 300
                    while got is None and time.monotonic() < deadline:
                        for key, payloads in t.drain_received().items():
                            if key == tid:
                                got = payloads[0]
                        if got is None:
                            if bar.failed():
                                raise ArmFailure(bar.failed())
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
                _role_call(bar, "consumer hand-off", receive)
                bar.set(f"h_done_{i}", repr(1e3 * (time.time() - t0)))
        bar.wait()
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
    if rank != 0:
        return {}
    tm = [float(bar.get(f"h_done_{i}")) for i in range(args.warmup, n_req)]
    sent = [json.loads(bar.get(f"h_sent_{i}")) for i in range(args.warmup, n_req)]
    raw = 2 * L * nblk * bs * H * D * 2
    return {
        "kv_transfer_ms_p50": round(statistics.median(tm), 3),
        "definition": "one TP channel's KV hand-off on its own (reference connector data path without vLLM: "
                      "compress, CompressedWire, NcclTransport send/recv, restore, decompress, inject), host "
                      "clock after device synchronisation, shared start to KV in the consumer's cache",
        "kv_send_ms_p50": round(statistics.median(x["sent_ms"] for x in sent), 3),
        "kv_payload_bytes_per_request": sent[0]["bytes"] * tp,
        "kv_raw_bytes_per_request": raw * tp,
        "compression_ratio": round(raw / sent[0]["bytes"], 3),
        "heads_per_channel": H,
        "data": "synthetic N(0,1) bf16 KV of the request's shape",
    }


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
