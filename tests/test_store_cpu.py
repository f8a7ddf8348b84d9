"""Prefix KV store on CPU: chained hashes, tiered LRU demotion to host and
disk, promotion on get, prefix lookup/save/load, compressed values, TP
layouts and metrics."""
import pytest
import torch

from kvserve_b200.store import (KVStoreConnector, RankLocalLayout, TieredKVPool, TPShardedLayout, block_hashes,
                                chunk_hashes)


def test_chained_hashes_identify_prefixes():
    a = block_hashes(list(range(64)), 16)
    b = block_hashes(list(range(48)) + [999] * 16, 16)
    assert len(a) == 4 and a[:3] == b[:3] and a[3] != b[3]
    assert block_hashes(list(range(64)), 16, extra=b"lora") != a
    assert chunk_hashes(a, 2) == [a[1], a[3]]


def test_pool_demotes_to_host_and_disk_and_promotes(tmp_path):
    pool = TieredKVPool(device_bytes=2 * 4096, host_bytes=4096, disk_dir=str(tmp_path), device="cpu")
    vals = {f"k{i}": torch.full((1024,), float(i)) for i in range(5)}   # 4 KB each
    for k, v in vals.items():
        pool.put(k, v)
    pool.flush()
    assert [pool.tier_of(f"k{i}") for i in range(5)] == ["disk", "disk", "host", "device", "device"]
    assert torch.equal(pool.get("k0"), vals["k0"])           # disk -> device
    assert pool.tier_of("k0") == "device" and pool.get("nope") is None
    text = __import__("prometheus_client").generate_latest(pool.registry).decode()
    assert 'kvs_store_hits_total{tier="disk"} 1.0' in text and "kvs_store_misses_total 1.0" in text
    pool.close()


@pytest.mark.parametrize("compressed", [False, True])
def test_connector_prefix_save_lookup_load(compressed):
    L, H, D, bs = 2, 4, 128, 16
    pool = TieredKVPool(device_bytes=1 << 30, host_bytes=1 << 30, device="cpu")
    cfg = None
    if compressed:
        cfg = {"enabled": True, "pipeline": ["transformer", "quantizer"],
               "transformer_config": {"transform_type": "hadamard"},
               "quantizer_config": {"hybrid_ratio": 0.0, "high_key_max_value": 254, "high_value_max_value": 254,
                                    "low_key_max_value": 254, "low_value_max_value": 254, "axis_key": "channel",
                                    "axis_value": "token", "split_type": "head"}}
    conn = KVStoreConnector(pool, bs, blocks_per_chunk=2, compression=cfg, num_kv_heads=H, head_size=D,
                            num_layers=L)
    torch.manual_seed(0)
    tokens = list(range(100))                     # 6 full blocks = 3 chunks (+4 tokens)
    kv = torch.randn(L, 2, 10, bs, H, D).to(torch.bfloat16)
    blocks = [3, 1, 4, 0, 5, 9, 2]
    assert conn.lookup(tokens) == 0
    assert conn.save(tokens, kv, blocks) == 3
    assert conn.lookup(tokens) == 96 and conn.lookup(tokens[:40]) == 32
    assert conn.lookup(tokens[:32] + [7] * 68) == 32
    dst = torch.zeros_like(kv)
    new_blocks = [8, 7, 6, 5, 4, 3, 2]
    assert conn.load(tokens, dst, new_blocks) == 96
    src = kv[:, :, blocks[:6]].float()
    got = dst[:, :, new_blocks[:6]].float()
    err = ((got - src).norm() / src.norm()).item()
    assert (err == 0.0) if not compressed else (err < 0.02)


def test_tp_sharded_layout_maps_head_ranges():
    lay = TPShardedLayout("m", tp_rank=1, tp_size=2, num_kv_heads=8, store_tp_size=4)
    assert lay.shards() == ["heads4-6", "heads6-8"]
    with pytest.raises(ValueError):
        TPShardedLayout("m", tp_rank=0, tp_size=4, num_kv_heads=8, store_tp_size=2)
    assert RankLocalLayout("m", 1, 2).shards() == ["tp1of2"]


def test_shared_pool_directory_is_seen_by_another_pool_and_pruned_oldest_first(tmp_path):
    """Two pools on one directory (two processes in production): a value
    put by one is found and read by the other; the directory's byte budget
    removes the oldest files first."""
    import time
    a = TieredKVPool(1 << 20, 1 << 20, disk_dir=str(tmp_path), device="cpu", shared=True, disk_bytes=3 * 6000)
    b = TieredKVPool(0, 0, disk_dir=str(tmp_path), device="cpu", shared=True)
    try:
        vals = {f"k{i}": torch.full((1024,), float(i)) for i in range(5)}   # ~5 KB files
        for k, v in vals.items():
            a.put(k, v)
            a.flush()
            time.sleep(0.02)
        assert b.contains("k4") and torch.equal(b.get("k4"), vals["k4"])
        assert not b.contains("k0") and not b.contains("k1")     # pruned, oldest first
        assert a.tier_of("k0") == "device"                        # still held in memory by its writer
    finally:
        a.close()
        b.close()
