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


def _cpu_runtimes(pipeline, layout="NHD", per_chunk=4, levels=None):
    from kvserve_b200.compression.runtime import create_runtime
    comp = {"enable-compression-pipeline": True, "pipeline": pipeline, "logical_blocks_per_chunk": per_chunk}
    comp.update(levels or {})
    cfg = CompressionConfig.from_extra_config({"compression": comp})
    specs = {f"l{i}": CacheSpec(i, 16, 4, 128, torch.bfloat16) for i in range(3)}
    plan = build_memory_plan(cfg, specs, num_layers=3, device="cpu")
    return (create_runtime(plan, layout, 1, "cpu", execution="encode"),
            create_runtime(plan, layout, 1, "cpu", execution="decode"))


def _cpu_caches(layout, fill, seed=5):
    g = torch.Generator().manual_seed(seed)
    shape = (2, 24, 16, 4, 128) if layout == "NHD" else (2, 24, 4, 16, 128)
    mk = (lambda: torch.randn(shape, generator=g)) if fill else (lambda: torch.zeros(shape))
    return {f"l{i}": mk().to(torch.bfloat16) for i in range(3)}


@pytest.mark.parametrize("layout", ["NHD", "HND"])
@pytest.mark.parametrize("pipeline", [["transformer", "quantizer"], ["transformer", "quantizer", "codec"]])
def test_cpu_runtime_round_trip_through_the_slot_api(layout, pipeline):
    """The runtime API on the CPU: encode a chunk of paged blocks (K and V
    parts) into a slot, move the payload into the peer's receive buffer,
    decode into other blocks; the result is the frame format's
    reconstruction (relative error of 4-bit symbols) and only the target
    blocks change."""
    enc, dec = _cpu_runtimes(pipeline, layout, levels={"high_key_num_levels": 16, "low_key_num_levels": 16,
                                                       "high_value_num_levels": 16, "low_value_num_levels": 16})
    src, dst = _cpu_caches(layout, True), _cpu_caches(layout, False)
    enc.bind_kv_caches(src)
    dec.bind_kv_caches(dst)
    assert enc.wire_profile == dec.wire_profile
    sb, db, valid = [3, 4, 5, 6], [10, 11, 12, 13], 4 * 16 - 5
    for part in (0, 1):
        r = enc.encode(0, {0: sb}, part, valid_tokens_by_group={0: valid})
        r.event.synchronize()
        n = r.codec_bytes
        dec.receive_buffer(1)[:n].copy_(r.payload[:n])
        dec.decode(1, {0: db}, part, codec_bytes=n, valid_tokens_by_group={0: valid}).synchronize()
    for name in src:
        s, d = src[name].float(), dst[name].float()
        tok = (lambda t, b: t[:, b].reshape(2, -1, 4, 128)) if layout == "NHD" else \
            (lambda t, b: t[:, b].permute(0, 1, 3, 2, 4).reshape(2, -1, 4, 128))
        a, b = tok(s, sb)[:, :valid], tok(d, db)[:, :valid]
        assert ((a - b).norm() / a.norm()) < 0.15
        assert tok(d, db)[:, valid:].abs().sum() == 0            # tail rows of the last block untouched
        others = [i for i in range(24) if i not in db]
        assert d[:, others].abs().sum() == 0


def test_cpu_runtime_frames_match_the_gpu_layout():
    """Each layer's frame sits at the same slot offset the GPU runtime uses
    and starts with the frame header (magic, layer, tokens)."""
    import struct
    from kvserve_b200.ops.kv_codec import FRAME_MAGIC
    enc, _ = _cpu_runtimes(["transformer", "quantizer"])
    enc.bind_kv_caches(_cpu_caches("NHD", True))
    enc.encode(0, {0: [0, 1]}, 0, valid_tokens_by_group={0: 32})
    arena = enc.slots[0].arena.numpy()
    for i in range(3):
        magic, _, layer, tokens = struct.unpack_from("<4I", arena, i * enc.layout.frame_stride)
        assert (magic, layer, tokens) == (FRAME_MAGIC, i, 32)


def test_cpu_runtime_slot_safety():
    """Slot bookkeeping of the runtime API: every encode bumps the slot's
    generation, a chunk larger than the plan is refused before any work,
    execution roles are enforced, and the wire profile names the layout."""
    enc, dec = _cpu_runtimes(["transformer", "quantizer"], per_chunk=2)
    enc.bind_kv_caches(_cpu_caches("NHD", True))
    dec.bind_kv_caches(_cpu_caches("NHD", False))
    g0 = enc.slots[0].generation
    enc.encode(0, {0: [0, 1]}, "key")
    enc.encode(0, {0: [0, 1]}, "value")
    assert enc.slots[0].generation == g0 + 2
    with pytest.raises(ValueError, match="more blocks"):
        enc.encode(0, {0: [0, 1, 2]}, 0)
    with pytest.raises(RuntimeError, match="encode only"):
        enc.decode(0, {0: [0, 1]}, 0)
    with pytest.raises(RuntimeError, match="decode only"):
        dec.encode(0, {0: [0, 1]}, 0)
    with pytest.raises(ValueError):
        enc.encode(0, {0: [0, 1]}, "both")
    assert enc.wire_profile.startswith("kvs-b200-frame-v1:") and enc.wire_profile == dec.wire_profile
    other, _ = _cpu_runtimes(["transformer", "quantizer"], per_chunk=4)
    other.bind_kv_caches(_cpu_caches("NHD", True))
    assert other.wire_profile != enc.wire_profile          # a different chunk geometry is another profile
