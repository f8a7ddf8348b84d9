"""Fixed-profile runtime round trips on the GPU (producer and consumer runtimes
in one process; a device copy stands in for the network)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(layout, pipeline, L=3, H=4, D=128, bs=16, nb=40, lbpc=4):
    from kvserve_b200.compression.runtime import CacheSpec, CompressionConfig, build_memory_plan, create_runtime
    cfg = CompressionConfig.from_extra_config({"compression": {
        "enable-compression-pipeline": True, "pipeline": pipeline, "logical_blocks_per_chunk": lbpc,
        "high_key_num_levels": 16, "low_key_num_levels": 16, "high_value_num_levels": 16,
        "low_value_num_levels": 16}})
    specs = {f"l{i}": CacheSpec(i, bs, H, D, torch.bfloat16) for i in range(L)}
    shape = (nb, H, bs, D) if layout == "HND" else (nb, bs, H, D)
    torch.manual_seed(0)
    src = {n: torch.randn((2,) + shape, dtype=torch.bfloat16, device="cuda") for n in specs}
    dst = {n: torch.zeros((2,) + shape, dtype=torch.bfloat16, device="cuda") for n in specs}
    plan = build_memory_plan(cfg, specs, num_layers=L, device="cuda")
    p = create_runtime(plan, layout, 1, "cuda")
    d = create_runtime(plan, layout, 1, "cuda")
    p.bind_kv_caches(src)
    d.bind_kv_caches(dst)
    assert p.wire_profile == d.wire_profile
    return p, d, src, dst


@pytest.mark.parametrize("layout", ["HND", "NHD"])
@pytest.mark.parametrize("pipeline", [["transformer", "quantizer", "codec"], ["transformer", "quantizer"], ["codec"]])
def test_runtime_round_trip(layout, pipeline):
    p, d, src, dst = _setup(layout, pipeline)
    blocks_src, blocks_dst = [5, 9, 2, 30], [1, 7, 3, 11]
    valid = 3 * 16 + 5  # partial last block
    for part in (0, 1):
        enc = p.encode(0, {0: blocks_src}, part, valid_tokens_by_group={0: valid})
        enc.event.synchronize()
        n = enc.codec_bytes
        d.receive_buffer(0)[:n].copy_(enc.payload[:n])  # the "network"
        ev = d.decode(0, {0: blocks_dst}, part, codec_bytes=n, u8_bytes=enc.u8_bytes,
                      valid_tokens_by_group={0: valid})
        ev.synchronize()
        d.check_status()
    tok = 1 if layout == "NHD" else 2
    for name in src:
        for part in (0, 1):
            a = src[name][part].index_select(0, torch.tensor(blocks_src, device="cuda"))
            b = dst[name][part].index_select(0, torch.tensor(blocks_dst, device="cuda"))
            a = a.movedim(tok, 1).reshape(-1, *a.movedim(tok, 1).shape[2:])[:valid].float()
            b = b.movedim(tok, 1).reshape(-1, *b.movedim(tok, 1).shape[2:])[:valid].float()
            err = ((a - b).norm() / a.norm()).item()
            if pipeline == ["codec"]:
                assert err == 0.0
            else:
                assert err < 0.15
