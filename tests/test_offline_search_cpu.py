"""Offline search and profile-library assembly on a small synthetic sample."""
import json

from kvserve_b200.compression.controller import OnlineController, ProfileLibrary
from kvserve_b200.offline_search.search import run, synthetic_kv
from kvserve_b200.offline_search.space import SearchPoint, enumerate_space


def test_space_validity_and_dominance():
    pts = enumerate_space(levels=(16, 8), ratios=(0.0, 0.5))
    assert all(p.is_valid() for p in pts)
    a = SearchPoint(True, 0.2, 16, 16, 8, 8)
    b = SearchPoint(True, 0.5, 12, 8, 6, 4)
    assert a.dominates_quality(b) and not b.dominates_quality(a)


def test_search_and_library_feed_the_controller(tmp_path):
    kv = synthetic_kv(layers=2, tokens=128, heads=4)
    out = run(str(tmp_path), kv, tolerances=(5.0,), budget=8, levels=(16, 8, 4), ratios=(0.0, 1.0))
    best = out["results"]["5.0"]["best"]
    base = out["results"]["baseline"]["accuracy"]
    assert best is not None and best["compression_ratio"] > 1.5 and best["accuracy"] >= base - 0.05
    lib = ProfileLibrary(tmp_path / "profile_library.json")
    assert lib.get_num_profiles() >= 1
    ctrl = OnlineController(lib, epsilon=0.0)
    prof, ctx = ctrl.select_profile(1e9, 100.0, 0.0, 1e12, base - 0.05)  # slow link: compression pays off
    assert prof is not None
    assert (tmp_path / "cr_cache.csv").exists()
    json.loads((tmp_path / "tolerance_5_results.json").read_text())


def test_cache_simulators_trade_ratio_for_error():
    import torch
    from kvserve_b200.offline_search.cache_sim import CacheGenSim, DuoAttentionSim, KIVISim, KVServeSim
    from kvserve_b200.offline_search.search import synthetic_kv
    kv = synthetic_kv(layers=2, tokens=256, heads=4)
    err = lambda r: ((r.float() - kv.float()).norm() / kv.float().norm()).item()  # noqa: E731
    r2, cr2 = KIVISim(bits=2, group=32, residual=64)(kv)
    r4, cr4 = KIVISim(bits=4, group=32, residual=64)(kv)
    assert cr2 > cr4 > 2.0 and err(r4) < err(r2) < 0.5
    rc, crc = CacheGenSim()(kv)
    assert crc > 2.0 and err(rc) < 0.5
    rd, crd = DuoAttentionSim(sparsity=0.5, sink=16, recent=32)(kv)
    assert 1.3 < crd < 2.0 and torch.equal(rd[:, :, :, -32:], kv[:, :, :, -32:])
    cfg = {"enabled": True, "pipeline": ["transformer", "quantizer"],
           "transformer_config": {"transform_type": "hadamard"},
           "quantizer_config": {"hybrid_ratio": 0.0, "high_key_max_value": 16, "high_value_max_value": 16,
                                "low_key_max_value": 16, "low_value_max_value": 16, "axis_key": "channel",
                                "axis_value": "token", "split_type": "head"}}
    rk, crk = KVServeSim(cfg, 4, 128, num_layers=2)(kv)
    assert crk > 1.5 and err(rk) < 0.2


def test_simulated_hf_cache_degrades_prefill_kv():
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM
    from kvserve_b200.offline_search.cache_sim import KIVISim, simulated_cache
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=256)
    model = LlamaForCausalLM(cfg).eval()
    ids = torch.randint(0, 128, (1, 96))
    with torch.no_grad():
        ref = model(ids, use_cache=True).past_key_values
        cache = simulated_cache(KIVISim(bits=2, group=16, residual=32), 2)
        model(ids, past_key_values=cache, use_cache=True)
    assert set(cache.ratios) == {0, 1} and all(r > 1.5 for r in cache.ratios.values())
    k_ref = ref.layers[0].keys if hasattr(ref, "layers") else ref.key_cache[0]
    k_sim = cache.layers[0].keys if hasattr(cache, "layers") else cache.key_cache[0]
    assert k_ref.shape == k_sim.shape and not torch.equal(k_ref, k_sim)


def test_kivi_and_cachegen_style_baselines_round_trip():
    """The PyTorch restatements of KIVI's group quantisation (keys per channel
    over token groups, values per token over channel groups) and of the
    CacheGen-style delta quantiser invert their own packing: the error is
    that of the quantiser (4 bits < 2 bits)."""
    import torch
    from kvserve_b200.offline_search.component_speed import kivi_compress, kivi_decompress
    g = torch.Generator().manual_seed(0)
    x = torch.randn(256, 4, 128, generator=g).bfloat16()
    errs = {}
    for per_channel in (True, False):
        for bits in (2, 4):
            y = kivi_decompress(*kivi_compress(x, bits, per_channel), bits, per_channel)
            y = y.reshape(256, 4, 128) if per_channel else y.reshape(256, 4, 128)
            errs[(per_channel, bits)] = float(((y.float() - x.float()) ** 2).mean())
    for pc in (True, False):
        assert errs[(pc, 4)] < 0.01 < errs[(pc, 2)] < 0.25


def _profile(k_levels, v_levels, enabled=True):
    with open("configs/compression/hadamard_k4v2_bitpack.json") as f:
        p = json.load(f)
    q = p["quantizer_config"]
    q["high_key_max_value"] = q["low_key_max_value"] = k_levels
    q["high_value_max_value"] = q["low_value_max_value"] = v_levels
    p["codec_config"]["bitpack_bits"] = max((k_levels - 1).bit_length(), (v_levels - 1).bit_length())
    p["enabled"] = enabled
    return p


def test_model_accuracy_evaluator_scores_profiles_through_a_language_model():
    """The reference's accuracy evaluator shape: the same model with its
    default cache and with the profile's restored prefill KV, scores
    normalised to the default (100 = unchanged)."""
    from kvserve_b200.offline_search.model_eval import ModelAccuracyEvaluator, synthetic_prompts, tiny_llama
    lm = tiny_llama(layers=2, hidden=128, heads=2, kv_heads=1, vocab=256)
    ev = ModelAccuracyEvaluator(lm, synthetic_prompts(2, 96, 256), new_tokens=8)
    assert ev.evaluate(_profile(16, 16, enabled=False)) == 100.0
    hi = ev.evaluate(_profile(254, 254))
    lo = ev.evaluate(_profile(4, 4))
    assert 0.0 <= lo <= hi <= 100.0 and hi >= 95.0
    assert ev.last["compression_ratio"] > 1.5


def test_search_runs_on_the_model_evaluator(tmp_path):
    from kvserve_b200.offline_search.model_eval import ModelAccuracyEvaluator, synthetic_prompts, tiny_llama
    lm = tiny_llama(layers=2, hidden=128, heads=2, kv_heads=1, vocab=256)
    ev = ModelAccuracyEvaluator(lm, synthetic_prompts(1, 64, 256), new_tokens=4)
    kv = synthetic_kv(layers=2, tokens=64, heads=1, dim=64)
    out = run(str(tmp_path), kv, tolerances=(50.0,), budget=4, levels=(16, 4), ratios=(0.0,),
              model_accuracy=ev.evaluate)
    assert 0.0 <= out["results"]["baseline"]["accuracy"] <= 1.0


def test_captured_model_kv_feeds_the_search(tmp_path):
    """KV captured from a language model's prefill ([L, 2, B, S, H, D]) is
    the sample the search and its evaluators take."""
    import torch
    from kvserve_b200.offline_search.model_eval import capture_kv, synthetic_prompts, tiny_llama
    lm = tiny_llama(layers=2, hidden=128, heads=2, kv_heads=1, vocab=256)
    kv = capture_kv(lm, synthetic_prompts(2, 64, 256))
    assert kv.shape == (2, 2, 2, 64, 1, 64) and kv.dtype == torch.bfloat16
    out = run(str(tmp_path), kv, tolerances=(5.0,), budget=4, levels=(16, 4), ratios=(0.0,))
    assert out["results"]["5.0"]["evaluated"] >= 1


def test_model_evaluator_scores_baseline_methods():
    """Baseline methods (KIVI, CacheGen restatements) go through the same
    language-model tasks as the profiles."""
    from kvserve_b200.offline_search.cache_sim import CacheGenSim, KIVISim
    from kvserve_b200.offline_search.model_eval import ModelAccuracyEvaluator, synthetic_prompts, tiny_llama
    lm = tiny_llama(layers=2, hidden=128, heads=2, kv_heads=1, vocab=256)
    ev = ModelAccuracyEvaluator(lm, synthetic_prompts(1, 96, 256), new_tokens=4)
    for sim in (KIVISim(bits=2, residual=16), CacheGenSim()):
        score = ev.evaluate_sim(sim)
        assert 0.0 <= score <= 100.0 and ev.last["compression_ratio"] > 1.5
