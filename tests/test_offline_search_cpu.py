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
