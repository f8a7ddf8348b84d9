"""The session-protocol connector loaded into the image's vLLM (0.22) through
``kv_connector_module_path``: a prefill engine and a decode engine of one
tiny dummy-weight Llama on one GPU (two GPUs when present).

The prefill engine runs the prompt with ``do_remote_decode`` and returns
the router parameters; the decode engine receives them, claims the prompt
as an asynchronous load, pulls it chunk by chunk (the prefill engine's
encode kernels store into the decode engine's CUDA-IPC receive arena, the
decode kernels write the request's paged blocks) and generates.  Checked:
both engines finish, the decode engine produces the requested tokens, and
the session rows show every chunk moved (send and receive COMPLETE).
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
PROMPT = [(5 * i + 11) % 1000 + 3 for i in range(150)]        # 10 blocks of 16 (the last one partial)
COMP = {"enable-compression-pipeline": True, "pipeline": ["transformer", "quantizer"],
        "logical_blocks_per_chunk": 4, "high_key_num_levels": 16, "low_key_num_levels": 16,
        "high_value_num_levels": 16, "low_value_num_levels": 16}


def _free_port():
    for base in range(43000, 60000, 41):
        try:
            s = socket.socket()
            s.bind(("127.0.0.1", base))
            s.close()
            return base
        except OSError:
            continue
    raise RuntimeError("no free port")


def _engine(q, role, model_dir, port, stats, params_q, done, dev):
    os.environ["VLLM_ENABLE_V1_MULTIPROCESSING"] = "0"
    os.environ["KVSERVE_SESSION_STATS_PATH"] = stats
    os.environ["CUDA_VISIBLE_DEVICES"] = str(dev)
    out = None
    try:
        from vllm import LLM, SamplingParams
        from vllm.config import KVTransferConfig
        from vllm.inputs import TokensPrompt
        producer = role == "producer"
        if not producer:
            # start once the prefill engine has built itself and run the
            # prompt (engines profiling memory at once on one GPU count each
            # other's allocations)
            params = params_q.get(timeout=600)
        kv = KVTransferConfig(kv_connector="SessionKVConnector",
                              kv_connector_module_path="kvserve_b200.connector.session_kv_connector",
                              kv_role="kv_producer" if producer else "kv_consumer", kv_ip="127.0.0.1",
                              kv_connector_extra_config={"session_port": port, "num_slots": 2, "compression": COMP})
        llm = LLM(model=model_dir, load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16",
                  max_model_len=512, enforce_eager=True, gpu_memory_utilization=0.2, seed=0,
                  enable_prefix_caching=False, kv_transfer_config=kv)
        prompt = [TokensPrompt(prompt_token_ids=PROMPT)]
        if producer:
            sp = SamplingParams(max_tokens=1, temperature=0.0, ignore_eos=True, detokenize=False,
                                extra_args={"kv_transfer_params": {"do_remote_decode": True,
                                                                   "transfer_id": "sess-vllm-0"}})
            res = llm.generate(prompt, sampling_params=sp, use_tqdm=False)
            params = res[0].kv_transfer_params
            params_q.put(params)
            # keep serving pulls until the decode engine is done
            if not done.wait(600):
                raise RuntimeError("the decode engine did not finish")
            out = ("ok", params)
        else:
            sp = SamplingParams(max_tokens=8, temperature=0.0, ignore_eos=True, detokenize=False,
                                extra_args={"kv_transfer_params": params})
            res = llm.generate(prompt, sampling_params=sp, use_tqdm=False)
            out = ("ok", list(res[0].outputs[0].token_ids))
    except BaseException:  # noqa: BLE001 - reported to the test
        import traceback
        out = ("error", traceback.format_exc()[-3000:])
    finally:
        if role == "consumer":
            done.set()
        q.put((role, out))
        q.close()
        q.join_thread()
        os._exit(0)


def test_vllm_session_connector_pulls_the_prompt_kv():
    pytest.importorskip("vllm")
    d = tempfile.mkdtemp(prefix="kvs_vllm_sess_")
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(TINY, f)
    stats = os.path.join(d, "sessions.jsonl")
    devs = (0, 1) if torch.cuda.device_count() > 1 else (0, 0)
    ctx = mp.get_context("spawn")
    q, params_q, done = ctx.Queue(), ctx.Queue(), ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_engine, args=(q, role, d, port, stats, params_q, done, dev))
             for role, dev in (("producer", devs[0]), ("consumer", devs[1]))]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in procs:
            role, out = q.get(timeout=900)
            res[role] = out
            if role == "producer" and out[0] != "ok":
                params_q.put({})       # unblock the consumer
    finally:
        done.set()
        for p in procs:
            p.join(30)
            if p.is_alive():
                p.kill()
    for role, (state, val) in res.items():
        assert state == "ok", f"{role}: {val}"
    params = res["producer"][1]
    assert params["do_remote_prefill"] and params["transfer_id"] == "sess-vllm-0"
    assert len(res["consumer"][1]) == 8
    rows = [json.loads(x) for x in open(stats)]
    recv = [r for r in rows if r["direction"] == "recv"]
    send = [r for r in rows if r["direction"] == "send"]
    assert recv and recv[0]["state"] == "COMPLETE" and recv[0]["chunks"] == recv[0]["total_chunks"] == 3, rows
    assert send and send[0]["state"] == "COMPLETE", rows
