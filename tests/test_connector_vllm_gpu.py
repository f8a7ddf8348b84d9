"""This framework's connector loaded into the image's vLLM (0.22) through
``kv_connector_module_path``, one GPU, KV over the transport's CUDA-IPC data
plane.

Three engines of one tiny dummy-weight Llama (vLLM's dummy loader seeds the
weights, so the engines hold identical weights):

* a producer (``kv_producer``) prefills the prompt and sends its KV;
* a consumer (``kv_consumer``) claims ``prompt_len - 1`` tokens from the
  connector, computes the last one and decodes;
* a reference engine with prefix caching runs the prompt twice; its second
  run computes only the last token against the cached KV of the first —
  the same arithmetic the consumer performs on the received KV.

With the uncompressed profile the consumer's greedy tokens equal the
reference's; with the K4/V2 profile (Hadamard + min-max + bit-packing) the
request completes with the requested number of tokens.
"""
import json
import multiprocessing as mp
import os
import socket
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu

TINY = {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 256,
        "intermediate_size": 512, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 64,
        "num_hidden_layers": 2, "vocab_size": 1024, "max_position_embeddings": 4096, "rope_theta": 10000.0,
        "rms_norm_eps": 1e-5, "hidden_act": "silu", "tie_word_embeddings": False, "torch_dtype": "bfloat16",
        "bos_token_id": 1, "eos_token_id": 2}
PROMPT = [(7 * i + 3) % 1000 + 3 for i in range(65)]     # 64 cached tokens + 1 computed
K4V2 = {"enabled": True, "pipeline": ["transformer", "quantizer", "codec"],
        "transformer_config": {"transform_type": "hadamard", "seed": 3237919422},
        "quantizer_config": {"model_name": "tiny", "hybrid_ratio": 0.0, "high_key_max_value": 16,
                             "high_value_max_value": 4, "low_key_max_value": 16, "low_value_max_value": 4,
                             "axis_key": "channel", "axis_value": "token", "split_type": "head"},
        "codec_config": {"codec_type": "bitpack", "bitpack_bits": 4}}


def _port_block():
    for base in range(42000, 60000, 37):
        try:
            s = socket.socket()
            s.bind(("127.0.0.1", base))
            s.close()
            return base
        except OSError:
            continue
    raise RuntimeError("no free port")


def _engine(q, role, model_dir, port, profile, max_tokens, ready=None):
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
    os.environ["KVSERVE_LOAD_TIMEOUT_S"] = "300"    # the producer may still be starting
    out = None
    try:
        from vllm import LLM, SamplingParams
        from vllm.config import KVTransferConfig
        from vllm.inputs import TokensPrompt
        kw = dict(model=model_dir, load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16",
                  max_model_len=512, enforce_eager=True, gpu_memory_utilization=0.2, seed=0)
        if role == "producer" and ready is not None:
            # vLLM sizes its KV cache from the memory it sees while profiling:
            # engines starting at the same time on one GPU count each other's
            # allocations, so the producer starts once the consumer is built
            if not ready.wait(300):
                raise RuntimeError("the consumer engine did not start")
        if role == "reference":
            llm = LLM(enable_prefix_caching=True, **kw)
        else:
            kv = KVTransferConfig(kv_connector="CompressedKVConnector",
                                  kv_connector_module_path="kvserve_b200.connector.compressed_kv_connector",
                                  kv_role="kv_producer" if role == "producer" else "kv_consumer",
                                  kv_rank=0 if role == "producer" else 1, kv_parallel_size=2, kv_ip="127.0.0.1",
                                  kv_port=port, kv_buffer_size=64 << 20,
                                  kv_connector_extra_config={"compression": profile, "data_plane": "ipc"})
            llm = LLM(enable_prefix_caching=False, kv_transfer_config=kv, **kw)
            if role == "consumer" and ready is not None:
                ready.set()
        sp = SamplingParams(max_tokens=max_tokens, temperature=0.0, ignore_eos=True, detokenize=False,
                            extra_args={"kv_transfer_params": {"transfer_id": "kvs-vllm-test-0"}})
        runs = 2 if role == "reference" else 1
        for _ in range(runs):
            res = llm.generate([TokensPrompt(prompt_token_ids=PROMPT)], sampling_params=sp, use_tqdm=False)
        out = ("ok", list(res[0].outputs[0].token_ids))
    except BaseException as exc:  # noqa: BLE001 - reported to the test
        import traceback
        out = ("error", traceback.format_exc()[-3000:])
    finally:
        q.put((role, out))
        q.close()
        q.join_thread()
        os._exit(0)


def _run(profile, max_tokens=8):
    d = tempfile.mkdtemp(prefix="kvs_vllm_tiny_")
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(TINY, f)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port_block()
    ready = ctx.Event()
    res = {}
    # the PD pair first (started one after the other), then the reference
    # engine on its own
    for roles in (("consumer", "producer"), ("reference",)):
        procs = [ctx.Process(target=_engine, args=(q, role, d, port, profile,
                                                   1 if role == "producer" else max_tokens, ready))
                 for role in roles]
        for p in procs:
            p.start()
        try:
            for _ in procs:
                role, out = q.get(timeout=600)
                res[role] = out
        finally:
            for p in procs:
                p.join(30)
                if p.is_alive():
                    p.kill()
    return res


def test_vllm_pd_raw_tokens_equal_prefix_cached_reference():
    pytest.importorskip("vllm")
    res = _run(None)
    for role, (state, val) in res.items():
        assert state == "ok", f"{role}: {val}"
    assert res["consumer"][1] == res["reference"][1]
    assert len(res["consumer"][1]) == 8


def test_vllm_pd_compressed_profile_completes():
    pytest.importorskip("vllm")
    res = _run(K4V2)
    for role in ("producer", "consumer"):
        state, val = res[role]
        assert state == "ok", f"{role}: {val}"
    assert len(res["consumer"][1]) == 8
