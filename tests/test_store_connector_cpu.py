"""The prefix-store vLLM connector on CPU: two engines (scheduler and worker
halves each, driven the way vLLM's scheduler and model runner call them)
share one store directory.  Engine A saves a prompt's KV chunk by chunk
after the forward that completes it; engine B finds the stored prefix,
claims it as external tokens and loads it into its own blocks — exactly
(raw) or within the codec's error (compressed) — skipping blocks it already
holds; a chunk that disappears between lookup and load comes back as
invalid blocks."""
import glob
import os
from types import SimpleNamespace as NS

import pytest
import torch

from kvserve_b200.connector.store_kv_connector import KVConnectorRole, StoreKVConnector

BS, BPC, NB, L, H, D = 16, 2, 40, 2, 2, 64
K4V4 = {"enabled": True, "pipeline": ["transformer", "quantizer", "codec"],
        "transformer_config": {"transform_type": "hadamard", "seed": 11},
        "quantizer_config": {"model_name": "tiny", "hybrid_ratio": 0.0, "high_key_max_value": 15,
                             "high_value_max_value": 15, "low_key_max_value": 15, "low_value_max_value": 15,
                             "axis_key": "channel", "axis_value": "token", "split_type": "head",
                             "num_layers": L, "num_kv_heads": H},
        "codec_config": {"codec_type": "bitpack", "bitpack_bits": 4}}


def _cfg(store_dir, compression=None):
    return NS(kv_transfer_config=NS(kv_connector_extra_config={
        "store": {"dir": store_dir, "device_bytes": 1 << 22, "host_bytes": 1 << 22, "blocks_per_chunk": BPC},
        "compression": compression}),
        cache_config=NS(block_size=BS), parallel_config=NS(tensor_parallel_size=1),
        model_config=NS(model="/models/tiny-llama", use_mla=False))


class Blocks:
    def __init__(self, ids):
        self.ids = ids

    def get_block_ids(self):
        return (self.ids,)


def _engine(store_dir, compression=None, seed=0, zero=False):
    g = torch.Generator().manual_seed(seed)
    caches = {f"model.layers.{i}.self_attn.attn":
              (torch.zeros if zero else (lambda *s, **k: torch.randn(*s, generator=g)))(2, NB, BS, H, D)
              .to(torch.bfloat16) for i in range(L)}
    sched = StoreKVConnector(_cfg(store_dir, compression), KVConnectorRole.SCHEDULER)
    work = StoreKVConnector(_cfg(store_dir, compression), KVConnectorRole.WORKER)
    work.register_kv_caches(caches)
    return sched, work, [caches[f"model.layers.{i}.self_attn.attn"] for i in range(L)]


def _so(new=()):
    return NS(scheduled_new_reqs=[NS(req_id=r, prompt_token_ids=p, block_ids=(b,), num_computed_tokens=c)
                                  for r, p, b, c, _ in new],
              num_scheduled_tokens={r: n for r, _, _, _, n in new},
              scheduled_cached_reqs=NS(req_ids=[], new_block_ids=[], num_computed_tokens=[], resumed_req_ids=set()))


def _step(sched, work, so):
    work.bind_connector_metadata(sched.build_connector_meta(so))
    work.start_load_kv(None)
    work.wait_for_save()
    work.clear_connector_metadata()


def _req(rid, prompt):
    return NS(request_id=rid, prompt_token_ids=prompt)


def _stack(layers, ids):
    return torch.stack([t[:, ids] for t in layers]).float()


@pytest.mark.parametrize("compressed", [False, True])
def test_second_engine_loads_the_stored_prefix(tmp_path, compressed):
    comp = K4V4 if compressed else None
    a_sched, a_work, a_kv = _engine(str(tmp_path), comp, seed=1)
    b_sched, b_work, b_kv = _engine(str(tmp_path), comp, zero=True)
    try:
        prompt = list(range(1000, 1100))                  # 100 tokens: 6 full blocks, 3 chunks of 32
        a_blocks = list(range(0, 7))
        assert a_sched.get_num_new_matched_tokens(_req("a1", prompt), 0) == (0, False)
        _step(a_sched, a_work, _so([("a1", prompt, a_blocks, 0, 100)]))
        assert a_work.stats["saved_chunks"] == 3
        a_work._store.pool.flush()
        assert len(glob.glob(os.path.join(str(tmp_path), "*.pt"))) == 3

        # engine B: same first 96 tokens, another tail
        prompt_b = prompt[:96] + list(range(5000, 5014))
        b_blocks = list(range(10, 17))
        req = _req("b1", prompt_b)
        assert b_sched.get_num_new_matched_tokens(req, 0) == (96, False)
        b_sched.update_state_after_alloc(req, Blocks(b_blocks), 96)
        _step(b_sched, b_work, _so([("b1", prompt_b, b_blocks, 96, 14)]))
        assert b_work.stats["loaded_tokens"] == 96 and not b_work.get_block_ids_with_load_errors()
        st = b_work.get_kv_connector_stats()            # vLLM's per-interval telemetry
        assert st.reduce() == {"loaded_tokens": 96, "saved_chunks": 0, "load_errors": 0}
        assert b_work.get_kv_connector_stats() is None
        assert a_work.get_kv_connector_stats().reduce()["saved_chunks"] == 3
        got, want = _stack(b_kv, b_blocks[:6]), _stack(a_kv, a_blocks[:6])
        if compressed:
            assert ((got - want).norm() / want.norm()) < 0.2
        else:
            assert torch.equal(got, want)
        assert _stack(b_kv, b_blocks[6:]).abs().sum() == 0    # the tail is computed, not loaded

        # a local prefix-cache hit of 2 blocks: only chunks 1 and 2 are copied
        blocks_c = list(range(20, 27))
        for t in b_kv:
            t[:, blocks_c[:2]] = 7
        req = _req("b2", prompt_b)
        assert b_sched.get_num_new_matched_tokens(req, 32) == (64, False)
        b_sched.update_state_after_alloc(req, Blocks(blocks_c), 64)
        _step(b_sched, b_work, _so())
        assert torch.all(_stack(b_kv, blocks_c[:2]) == 7)
        assert torch.equal(_stack(b_kv, blocks_c[2:6]), _stack(b_kv, b_blocks[2:6]))

        # the whole prompt stored: the last token is still computed
        assert b_sched.get_num_new_matched_tokens(_req("b3", prompt[:96]), 0) == (64, False)
    finally:
        a_work.shutdown()
        b_work.shutdown()
        a_sched.shutdown()
        b_sched.shutdown()


def test_chunk_missing_at_load_time_is_reported(tmp_path):
    a_sched, a_work, _ = _engine(str(tmp_path), seed=2)
    b_sched, b_work, _ = _engine(str(tmp_path), zero=True)
    try:
        prompt = list(range(100))
        _step(a_sched, a_work, _so([("a1", prompt, list(range(7)), 0, 100)]))
        a_work._store.pool.flush()
        req = _req("b1", prompt)
        assert b_sched.get_num_new_matched_tokens(req, 0) == (96, False)
        b_sched.update_state_after_alloc(req, Blocks(list(range(10, 17))), 96)
        files = sorted(glob.glob(os.path.join(str(tmp_path), "*.pt")), key=os.path.getmtime)
        # drop the last chunk written (chunk 2: blocks 14, 15)
        keys = b_work._store._keys(prompt)
        os.remove(b_work._store.pool._path(keys[2]))
        _step(b_sched, b_work, _so())
        assert b_work.stats["loaded_tokens"] == 64
        assert b_work.get_block_ids_with_load_errors() == {14, 15}
        assert len(files) == 3
    finally:
        a_work.shutdown()
        b_work.shutdown()
        b_sched.shutdown()


def test_sliding_window_and_hybrid_layouts_are_refused(tmp_path):
    class SlidingWindowSpec:                 # the name of vLLM's sliding-window spec
        sliding_window, block_size = 4096, BS

    class FullAttentionSpec:
        sliding_window, block_size = None, BS

    def groups(*specs):
        return NS(kv_cache_groups=[NS(kv_cache_spec=s()) for s in specs])

    with pytest.raises(ValueError, match="sliding-window"):
        StoreKVConnector(_cfg(str(tmp_path)), KVConnectorRole.SCHEDULER, groups(SlidingWindowSpec))
    with pytest.raises(ValueError, match="one KV-cache group"):
        StoreKVConnector(_cfg(str(tmp_path)), KVConnectorRole.SCHEDULER, groups(FullAttentionSpec, SlidingWindowSpec))
    StoreKVConnector(_cfg(str(tmp_path)), KVConnectorRole.SCHEDULER, groups(FullAttentionSpec)).shutdown()
