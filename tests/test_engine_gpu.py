"""The standalone PD engine on one GPU (colocated prefill + decode)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _engine(profile, max_prompt=255, max_new=8, graphs=True, model="tiny-gqa"):
    from kvserve_b200.engine.pd import PDEngine
    from kvserve_b200.models.config import get_config
    from kvserve_b200.parallel.context import ParallelContext
    return PDEngine(get_config(model), ParallelContext(), profile, max_prompt=max_prompt, max_new_tokens=max_new,
                    use_graphs=graphs)


def test_raw_handoff_reproduces_prefill_kv():
    """With the raw profile the decode-side paged cache must hold exactly the
    K/V the prefill computed."""
    from kvserve_b200.engine.transfer import TransferProfile
    eng = _engine(TransferProfile.raw())
    T = 200
    ids = torch.randint(0, eng.cfg.vocab, (T,), dtype=torch.int32)
    # run prefill+handoff but keep the blocks: allocate manually through generate, then inspect
    res = eng.generate(ids, 4)
    assert len(res.tokens) == 4
    # re-run the hand-off path directly and compare the cache with the prefill buffers
    blocks = eng.kv.allocate(T)
    table = eng.kv.block_table(blocks, eng.max_blocks)
    Tx = T - 1
    dev_ids = ids.cuda()
    eng.seq += 1

    def hook(l):
        eng.xfer.encode(l, eng.k_buf[l, :Tx], eng.v_buf[l, :Tx], eng.sender.frame_ptr(0, l), 0, eng.seq)
        eng.xfer.ingest_layer(l, Tx, eng.sender.frame_ptr(0, l), eng.kv.cache, table, eng.status, eng.seq)

    eng.model.prefill(dev_ids[:Tx], eng.positions[:Tx], eng.k_buf, eng.v_buf, layer_hook=hook)
    torch.cuda.synchronize()
    bs = eng.block_size
    got = eng.kv.cache[:, :, torch.tensor(blocks).cuda().long()].reshape(eng.cfg.num_layers, 2, -1, eng.model.hkv,
                                                                         eng.model.D)[:, :, :Tx]
    assert torch.equal(got[:, 0], eng.k_buf[:, :Tx])
    assert torch.equal(got[:, 1], eng.v_buf[:, :Tx])
    eng.kv.release(blocks)
    eng.close()


def test_first_token_matches_full_prefill_raw():
    from kvserve_b200.engine.transfer import TransferProfile
    eng = _engine(TransferProfile.raw())
    T = 180
    ids = torch.randint(0, eng.cfg.vocab, (T,), dtype=torch.int32)
    res = eng.generate(ids, 3)
    # the first token is the prefill's own greedy sample; the second comes from
    # the decode step over the handed-off KV and must equal a full prefill of
    # prompt + first token followed by greedy sampling
    kb = torch.empty((eng.cfg.num_layers, T + 1, eng.model.hkv, eng.model.D), dtype=torch.bfloat16, device="cuda")
    vb = torch.empty_like(kb)
    pos = torch.arange(T + 1, dtype=torch.int32, device="cuda")
    tok0 = eng.model.prefill(ids.cuda(), pos[:T], kb, vb, sample=True)
    assert int(tok0.item()) == res.tokens[0]
    ext = torch.cat([ids, torch.tensor([res.tokens[0]], dtype=torch.int32)]).cuda()
    tok1 = eng.model.prefill(ext, pos, kb, vb, sample=True)
    assert int(tok1.item()) == res.tokens[1]
    eng.close()


def test_compressed_handoff_generates_and_graph_matches_eager():
    from kvserve_b200.engine.transfer import TransferProfile
    prof = TransferProfile(compressed=True, hybrid_ratio=0.5, key_levels=(16, 16), value_levels=(16, 16))
    ids = torch.randint(0, 4096, (255,), dtype=torch.int32)
    a = _engine(prof, graphs=True)
    ra = a.generate(ids, 8)
    a.close()
    b = _engine(prof, graphs=False)
    rb = b.generate(ids, 8)
    b.close()
    assert ra.tokens == rb.tokens
    assert ra.timing.payload_bytes < ra.timing.raw_bytes / 3.5
    assert ra.timing.first_token > 0 and ra.timing.launches > 0
