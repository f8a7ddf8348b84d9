"""CPU tests of the modular compression library (no GPU needed)."""
import json
import math

import numpy as np
import pytest
import torch


def synthetic_kv(layers=2, tokens=256, heads=4, dim=128, seed=0):
    """values N(0,1); keys N(0,1) with 4 outlier channels per head x8."""
    g = torch.Generator().manual_seed(seed)
    kv = torch.randn((layers, 2, 1, tokens, heads, dim), generator=g)
    ch = torch.randperm(dim, generator=g)[:4]
    kv[:, 0, :, :, :, ch] *= 8
    return kv.to(torch.bfloat16)


CFG0 = {
    "enabled": True,
    "pipeline": ["transformer", "quantizer", "codec"],
    "transformer_config": {"transform_type": "hadamard", "seed": 3237919422},
    "quantizer_config": {"model_name": "synthetic", "hybrid_ratio": 0.0, "high_key_max_value": 15,
                         "high_value_max_value": 15, "low_key_max_value": 15, "low_value_max_value": 15,
                         "axis_key": "channel", "axis_value": "token", "split_type": "head",
                         "num_layers": 2, "num_kv_heads": 4},
    "codec_config": {"codec_type": "bitpack", "bitpack_bits": 4},
}


def test_config0_round_trip_ratio_and_mse():
    from kvserve_b200.compression.adapter import KVCompressionAdapter
    kv = synthetic_kv()
    ad = KVCompressionAdapter(CFG0, num_kv_heads=4, head_size=128, num_layers=2)
    c = ad.compress(kv, "req-0")
    assert c is not None and c.metadata["codec_applied"]
    out = ad.decompress(c)
    assert out.shape == kv.shape
    ratio = c.original_size / c.compressed_size
    mse = (out.float() - kv.float()).pow(2).mean().item()
    assert 3.9 < ratio < 4.0
    # 4-bit min-max after Hadamard: MSE well below the signal power
    assert mse < 0.05 * kv.float().pow(2).mean().item()


def test_bitpack_cpu_format_and_round_trip():
    from kvserve_b200.compression.codec.bitpack import BitPackCodec
    x = torch.tensor([1, 2, 3, 0, 7, 5, 6, 4, 2], dtype=torch.uint8)
    c = BitPackCodec(bitpack_bits=3)
    enc = c.encode(x)
    raw = enc.numpy().tobytes()
    assert raw[:4] == (0x0150424B).to_bytes(4, "little") and raw[4] == 3 and raw[5:8] == b"\0\0\0"
    assert int.from_bytes(raw[8:16], "little") == 9 and len(raw) == 16 + math.ceil(9 * 3 / 8)
    # LSB-first: symbols 1,2 -> bits 001 010 -> byte0 low bits 0b010001
    assert raw[16] & 0x3F == 0b010001
    dec = c.decode(enc, "uint8", [9], "cpu")
    assert torch.equal(dec, x)
    with pytest.raises(ValueError):
        c.encode(torch.tensor([9], dtype=torch.uint8))


@pytest.mark.parametrize("n", [1, 100, 16384, 40000])
def test_lossless_round_trip(n):
    from kvserve_b200.compression.codec.lossless import encode_bytes, decode_bytes
    rng = np.random.default_rng(n)
    data = rng.integers(0, 16, n, dtype=np.uint8)
    data[: n // 3] = 0
    enc = encode_bytes(data)
    assert np.array_equal(decode_bytes(enc), data)
    if n >= 16384:
        assert len(enc) < n * 0.75  # 4-bit symbols: upper bit planes are zero


def test_wire_round_trip_with_coalesced_aux():
    from kvserve_b200.compression.adapter import KVCompressionAdapter
    from kvserve_b200.compression.wire import build_wire, restore_from_wire, AUX_PLACEHOLDER
    kv = synthetic_kv()
    ad = KVCompressionAdapter(CFG0, num_kv_heads=4, head_size=128, num_layers=2)
    c = ad.compress(kv, "req-w")
    w = build_wire(c, max_chunk_bytes=1000)
    assert w.meta["body_mode"] == "byte_chunks" and len(w.aux_tensors) == 1
    assert w.meta["aux_layout"]["mode"] == "coalesced_bytes"
    txt = json.dumps(w.meta)
    assert AUX_PLACEHOLDER in txt
    import msgpack
    meta2 = msgpack.unpackb(msgpack.packb(w.meta), strict_map_key=False)
    w.meta = meta2
    r = restore_from_wire(w)
    out = ad.decompress(r)
    ref = ad.decompress(c)
    assert torch.equal(out, ref)


def test_fused_normalisation_keeps_seed_and_rejects_conflicts():
    from kvserve_b200.compression.adapter import KVCompressionAdapter as A
    cfg = {"pipeline": ["transformer", "quantizer", "codec"], "transformer_config": {"transform_type": "hadamard",
           "seed": 77}, "quantizer_config": {"impl": "tilelang_fused"}, "codec_config": {"codec_type": "bitpack"}}
    n = A.normalize_config(cfg)
    assert n["pipeline"] == ["quantizer", "codec"] and n["quantizer_config"]["base_seed"] == 77
    bad = dict(cfg, quantizer_config={"impl": "tilelang_fused", "base_seed": 78})
    with pytest.raises(ValueError):
        A.normalize_config(bad)
    with pytest.raises(ValueError):
        A.normalize_config(dict(cfg, transformer_config={"transform_type": "dct"}))


def test_fused_quantizer_cpu_round_trip():
    from kvserve_b200.compression.adapter import KVCompressionAdapter
    cfg = {"pipeline": ["transformer", "quantizer", "codec"],
           "transformer_config": {"transform_type": "hadamard", "seed": 5},
           "quantizer_config": {"impl": "tilelang_fused", "hybrid_ratio": 0.5, "model_name": "synthetic",
                                "num_layers": 2, "num_kv_heads": 4, "low_key_max_value": 16, "high_key_max_value": 16,
                                "low_value_max_value": 16, "high_value_max_value": 16},
           "codec_config": {"codec_type": "bitpack", "bitpack_bits": 4}}
    kv = synthetic_kv(tokens=64)
    ad = KVCompressionAdapter(cfg, num_kv_heads=4, head_size=128, num_layers=2)
    c = ad.compress(kv, "r")
    out = ad.decompress(c)
    err = (out.float() - kv.float()).norm() / kv.float().norm()
    assert err < 0.15


@pytest.mark.parametrize("kind", ["dct", "haar"])
def test_orthogonal_transform_inverts(kind):
    from kvserve_b200.compression.transformer import KVServeTransformer
    t = KVServeTransformer(transform_type=kind, seed=13107)
    x = torch.randn(2, 3, 16, 4, 128)
    y = t.transform(1, x)
    z = t.inverse(1, y)
    assert torch.allclose(z, x, atol=1e-4)
    assert not torch.allclose(y, x)


def test_centered_codebook_round_trip():
    from kvserve_b200.compression.quantizer import CenteredCodebookQuantizer
    from kvserve_b200.compression.quantizer.centered_codebook import lloyd_max_gaussian
    c2 = lloyd_max_gaussian(1)
    assert abs(abs(c2[0]) - math.sqrt(2 / math.pi)) < 1e-6
    q = CenteredCodebookQuantizer(key_bits=3, value_bits=3, group_size=32, scale_refinements=1)
    x = torch.randn(2, 2, 40, 4, 64)
    sym, meta = q.quantize(0, x)
    assert int(sym.max()) < 8
    y = q.dequantize(0, sym, meta)
    rel = ((y - x).norm() / x.norm()).item()
    assert rel < 0.3


def test_hybrid_quantizer_head_split_and_tp_slice():
    from kvserve_b200.compression.quantizer import KVServeQuantizer
    q = KVServeQuantizer(model_name="Llama-3.1-8B-Instruct", hybrid_ratio=0.5, tensor_parallel_size=2, tp_rank=1)
    assert q.head_scores.shape == (32, 8)
    m = q.head_mask(4)
    assert m.shape == (32, 4) and torch.equal(m, q.head_scores_mask[:, 4:8])
    x = torch.randn(2, 1, 16, 4, 128, dtype=torch.bfloat16)
    sym, meta = q.quantize(3, x)
    back = q.dequantize(3, sym, meta)
    assert back.shape == x.shape
    assert ((back.float() - x.float()).norm() / x.float().norm()) < 0.2


def test_signs_match_reference_generator_semantics():
    from kvserve_b200.compression.heads import rademacher_signs, pack_sign_bits
    s = rademacher_signs(3237919422, 2, 3, 128)
    g = torch.Generator().manual_seed(3237919422 ^ (2 << 16) ^ 1)
    ref = torch.randint(0, 2, (128,), generator=g, dtype=torch.int8).float() * 2 - 1
    assert torch.equal(s[1], ref)
    bits = pack_sign_bits(s)
    assert bits.shape == (3, 4)
    neg = [(int(bits[1, d // 32]) >> (d % 32)) & 1 for d in range(128)]
    assert neg == [(1 if v < 0 else 0) for v in ref.tolist()]


def test_controller_selects_and_learns(tmp_path):
    from kvserve_b200.compression.controller import OnlineController, ProfileLibrary, AnalyticalModel, Profile
    import random
    lib = {"library_metadata": {"model_name": "m"}, "accuracy_buckets": [{
        "bucket_id": 0, "acc_range": [0.0, 1.01],
        "bandwidth_intervals": [{"interval_id": 0, "x_range": [0.0, 1.0], "candidate_profile_ids": ["a", "b"]}],
        "pareto_profiles": [
            {"profile_id": "a", "compression_config": {"x": 1}, "performance_metrics":
             {"compression_ratio": 4.0, "harmonic_speed_mbps": 20000.0}, "quality_metrics": {"accuracy": 0.99}},
            {"profile_id": "b", "compression_config": {"x": 2}, "performance_metrics":
             {"compression_ratio": 8.0, "harmonic_speed_mbps": 10000.0}, "quality_metrics": {"accuracy": 0.95}}]}]}
    p = tmp_path / "lib.json"
    p.write_text(json.dumps(lib))
    ctrl = OnlineController(ProfileLibrary(p), epsilon=0.0, rng=random.Random(0))
    prof, ctx = ctrl.select_profile(1e9, 3125.0, 10.0, 1e9, 0.9)   # 25 Gbps
    assert prof is not None and ctx["action"] == "exploit"
    # at 400 Gbps (50 GB/s) neither profile beats the raw link (Theorem 1)
    none, c2 = ctrl.select_profile(1e9, 50000.0, 10.0, 1e9, 0.9)
    assert none is None and c2["reason"] == "no_benefit"
    ctrl.update(ctx, ctx["T_hat"] + 100.0)
    assert ctrl.bandit.get_residual(0, 0, prof.profile_id) == pytest.approx(20.0)
    ctrl.save_state(str(tmp_path / "b.json"))
    c3 = OnlineController(ProfileLibrary(p))
    c3.load_state(str(tmp_path / "b.json"))
    assert c3.bandit.get_stats(0, 0, prof.profile_id) == (1, pytest.approx(20.0))
    m = AnalyticalModel("reference")
    pa = Profile.from_dict(lib["accuracy_buckets"][0]["pareto_profiles"][0])
    assert m.predict_latency(pa, 1048576, 1.0, 0.0) == pytest.approx(1e3 / 20000 + 4e3)


@pytest.mark.parametrize("name", ["original_top_lc", "original_top_nvcomp", "dct_centered_bitpack",
                                  "haar_centered_bitpack", "hadamard_k4v2_bitpack"])
def test_shipped_profiles_round_trip(name):
    import json
    import os
    from kvserve_b200.compression.adapter import KVCompressionAdapter
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    with open(os.path.join(root, "configs", "compression", f"{name}.json")) as f:
        cfg = json.load(f)
    torch.manual_seed(0)
    kv = torch.randn(2, 2, 1, 64, 8, 128).to(torch.bfloat16)
    ad = KVCompressionAdapter(cfg, 8, 128, num_layers=2)
    c = ad.compress(kv, "r")
    assert c is not None and c.original_size / c.compressed_size > 2.0
    rec = ad.decompress(c)
    err = ((rec.float() - kv.float()).norm() / kv.float().norm()).item()
    assert rec.shape == kv.shape and err < 0.6


def test_fidelity_synthetic_kv_and_error_stats():
    from kvserve_b200.engine.fidelity import error_stats, synthetic_kv
    kv = synthetic_kv(2, 64, 4, 128, seed=0)
    assert kv.shape == (2, 2, 64, 4, 128) and kv.dtype == torch.bfloat16
    # keys carry 4 outlier channels x8: their power dwarfs the others
    kp = kv[:, 0].float().pow(2).mean(dim=(0, 1, 2))
    assert (kp > 16).sum() == 4
    st = error_stats(kv, torch.zeros_like(kv))
    assert abs(st["rel_mse"] - 1.0) < 1e-6 and abs(st["v_rel_mse"] - 1.0) < 1e-6
    assert error_stats(kv, kv)["mse"] == 0.0


def test_hadamard_bf16_kind_round_trips_and_differs_from_fp32_only_by_rounding():
    from kvserve_b200.compression.transformer.kvserve_transformer import KVServeTransformer, registered_transforms
    assert "hadamard_bf16" in registered_transforms()
    g = torch.Generator().manual_seed(5)
    layer = torch.randn((2, 3, 16, 4, 128), generator=g).to(torch.bfloat16)
    ref = KVServeTransformer(transform_type="hadamard", seed=77)
    stg = KVServeTransformer(transform_type="hadamard_bf16", seed=77)
    a, b = ref.transform(3, layer).float(), stg.transform(3, layer).float()
    assert not torch.equal(a, b)                      # per-stage rounding changes some values
    assert (a - b).abs().max() <= 0.05 * a.abs().max()
    back = stg.inverse(3, stg.transform(3, layer)).float()
    assert ((back - layer.float()).norm() / layer.float().norm()) < 0.02


def test_config0_end_to_end_over_two_gloo_processes():
    """The CPU benchmark configuration as a whole: compress the seeded sample,
    send the real wire bundle from a producer process to a consumer process
    over the credit transport's gloo data plane, decompress there, report
    CR and reconstruction error."""
    from kvserve_b200.engine.config0 import run
    r = run()
    assert r["error"] is None, r["error"]
    assert r["transferred"] and 3.9 < r["compression_ratio"] < 4.0 and r["wire_ratio"] > 3.8
    assert r["mse"] < 0.05 * r["signal_power"] and r["relative_error"] < 0.2
