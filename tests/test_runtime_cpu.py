"""Fixed-profile runtime API v1: configuration, head selection, memory plan (CPU)."""
import numpy as np
import pytest
import torch

from kvserve_b200.compression.runtime import API_VERSION, CacheSpec, CompressionConfig, build_memory_plan
from kvserve_b200.compression.runtime.scores import build_head_selection


def test_config_public_keys_and_validation():
    assert API_VERSION == 1
    assert not CompressionConfig.from_extra_config({}).enabled
    c = CompressionConfig.from_extra_config({"compression": {"enable-compression-pipeline": True,
                                                             "logical_blocks_per_chunk": 64}})
    assert c.enabled and c.transport == "compression" and c.logical_blocks_per_chunk == 64
    agg = CompressionConfig.from_extra_config({"raw_agg": True, "compression": {"enable-compression-pipeline": True}})
    assert agg.is_raw_aggregate and agg.pipeline == ("aggregate",) and agg.slot_count == 2
    for bad in ({"high_key_num_levels": 1}, {"pipeline": ["codec", "quantizer"]}, {"codec": "zstd"},
                {"hybrid_ratio": 1.5}, {"slot_count": 0}):
        with pytest.raises(ValueError):
            CompressionConfig.from_extra_config({"compression": {"enable-compression-pipeline": True, **bad}})
    with pytest.raises(ValueError):
        CompressionConfig.from_extra_config({"raw_aggregate": {"slots": 3}})


def _specs(L=4, H=2, D=128, bs=16):
    return {f"model.layers.{i}.attn": CacheSpec(i, bs, H, D, torch.bfloat16) for i in range(L)}


def test_head_selection_global_argsort_and_tp_slices():
    scores = np.array([[0.1, 0.9, 0.5, 0.3], [0.2, 0.8, 0.05, 0.7]], dtype=np.float32)
    cfg = CompressionConfig(enabled=True, split_type="head", hybrid_ratio=0.5)
    specs = {"a": CacheSpec(0, 16, 2, 128, torch.bfloat16), "b": CacheSpec(1, 16, 2, 128, torch.bfloat16)}
    s0 = build_head_selection(specs, cfg, tp_rank=0, tp_size=2, scores=scores)
    s1 = build_head_selection(specs, cfg, tp_rank=1, tp_size=2, scores=scores)
    # lowest 4 of 8: (1,2)=0.05, (0,0)=0.1, (1,0)=0.2, (0,3)=0.3
    assert s0.local_orders[0] == (0, 1) and s0.low_counts[0] == 1
    assert s1.local_orders[0] == (1, 0) and s1.low_counts[0] == 1
    assert s0.low_counts[1] == 1 and s1.low_counts[1] == 1 and s1.local_orders[1] == (0, 1)
    # replicated KV heads: 2 score columns, TP 4, one local head
    specs1 = {"a": CacheSpec(0, 16, 1, 128, torch.bfloat16)}
    r3 = build_head_selection(specs1, cfg, tp_rank=3, tp_size=4, scores=scores)
    assert r3.local_orders[0] == (0,)


def test_memory_plan_is_bounded_and_layer_split():
    cfg = CompressionConfig.from_extra_config({"compression": {"enable-compression-pipeline": True,
                                                               "logical_blocks_per_chunk": 8, "slot_count": 3}})
    plan = build_memory_plan(cfg, _specs(L=6), blocks_per_logical=1, num_layers=6)
    assert plan.layout.chunk_tokens == 128
    assert plan.reserved_bytes >= 3 * plan.slot_bytes
    lows = [e.n_low for e in plan.layout.layers]
    assert lows == [0, 0, 0, 0, 2, 2]   # split_type="layer": last round(0.33 * 6) layers low
    with pytest.raises(ValueError):
        build_memory_plan(cfg, {"x": CacheSpec(0, 16, 2, 128, torch.float16)})
