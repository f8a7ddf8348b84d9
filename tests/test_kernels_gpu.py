"""Numerics of the sm_100a kernels against plain PyTorch fp32 references."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from kvserve_b200 import ops
    return ops


def _rel_err(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 520, 136), (1024, 1024, 1024), (8192, 4096, 512),
                                   (17, 4096, 4096), (2048, 6144, 4096), (2200, 1280, 256)])
def test_gemm_tcgen05(M, N, K):
    ops = _ops()
    torch.manual_seed(0)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    c = ops.gemm(a, b)
    ops.check_device_status()
    ref = a.float() @ b.float().T
    assert _rel_err(c, ref) < 1e-2


@pytest.mark.parametrize("M,I,K", [(9, 256, 128), (300, 1024, 512), (4096, 3584, 4096)])
def test_gemm_silu_fused_epilogue(M, I, K):
    ops = _ops()
    torch.manual_seed(1)
    a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    g = torch.randn(I, K, device="cuda", dtype=torch.bfloat16) / math.sqrt(K)
    u = torch.randn(I, K, device="cuda", dtype=torch.bfloat16) / math.sqrt(K)
    w = ops.interleave_gate_up(g, u)
    y = ops.gemm_silu(a, w)
    ops.check_device_status()
    ref = torch.nn.functional.silu(a.float() @ g.float().T) * (a.float() @ u.float().T)
    assert _rel_err(y, ref) < 1e-2
    # the unfused path on the same interleaved layout (decode-size batches)
    y2 = ops.silu_mul(ops.gemm(a, w), block=ops.GATE_UP_BLOCK)
    assert _rel_err(y2, ref) < 1e-2


@pytest.mark.parametrize("T,Hq,Hkv,bias", [(300, 32, 8, False), (129, 28, 4, True), (1024, 8, 2, False)])
def test_gemm_qkv_rope_matches_unfused(T, Hq, Hkv, bias):
    ops = _ops()
    torch.manual_seed(2)
    K = 512
    N = (Hq + 2 * Hkv) * 128
    a = torch.randn(T, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) / math.sqrt(K)
    b = torch.randn(N, device="cuda", dtype=torch.bfloat16) if bias else None
    pos = torch.randperm(4096, device="cuda")[:T].to(torch.int32)
    inv = 1.0 / (500000.0 ** (torch.arange(0, 128, 2, dtype=torch.float64) / 128))
    ang = torch.outer(torch.arange(4096, dtype=torch.float64), inv)
    cs = torch.cat([ang.cos(), ang.sin()], -1).float().cuda()
    kd = torch.empty(T, Hkv, 128, device="cuda", dtype=torch.bfloat16)
    vd = torch.empty_like(kd)
    got = ops.gemm_qkv_rope(a, w, Hq, Hkv, pos, cs, bias=b, k_dst=kd, v_dst=vd)
    ops.check_device_status()
    ref = ops.gemm(a, w, bias=b)
    kr, vr = torch.empty_like(kd), torch.empty_like(vd)
    ops.rope_qkv(ref, Hq, Hkv, 128, pos, cs, kr, vr)
    assert _rel_err(got, ref) < 1e-2
    assert _rel_err(kd, kr) < 1e-2 and torch.equal(vd, got[:, (Hq + Hkv) * 128:].reshape(T, Hkv, 128))
    assert torch.equal(kd, got[:, Hq * 128:(Hq + Hkv) * 128].reshape(T, Hkv, 128))


def test_gemm_residual():
    ops = _ops()
    a = torch.randn(256, 512, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(768, 512, device="cuda", dtype=torch.bfloat16)
    r = torch.randn(256, 768, device="cuda", dtype=torch.bfloat16)
    c = ops.gemm(a, b, residual=r)
    ref = a.float() @ b.float().T + r.float()
    assert _rel_err(c, ref) < 1e-2


@pytest.mark.parametrize("M", [1, 2, 5, 8])
@pytest.mark.parametrize("N,K", [(4096, 4096), (1000, 14336), (128256, 4096)])
def test_gemv(M, N, K):
    ops = _ops()
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
    y = ops.gemv(x, w)
    ref = x.float() @ w.float().T
    assert _rel_err(y, ref) < 1e-2


def test_rmsnorm_and_residual():
    ops = _ops()
    x = torch.randn(37, 4096, device="cuda", dtype=torch.bfloat16)
    r = torch.randn(37, 4096, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(4096, device="cuda", dtype=torch.bfloat16)
    r_ref = (x.float() + r.float()).bfloat16().float()
    ref = (r_ref * torch.rsqrt(r_ref.pow(2).mean(-1, keepdim=True) + 1e-5)).bfloat16().float() * w.float()
    r2 = r.clone()
    y = ops.rmsnorm(x, w, 1e-5, residual=r2)
    assert torch.equal(r2.float(), r_ref)
    assert _rel_err(y, ref) < 1e-2
    y2 = ops.rmsnorm(x, w, 1e-5)
    ref2 = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-5)).bfloat16().float() * w.float()
    assert _rel_err(y2, ref2) < 1e-2


def _rope_cache(max_pos, d, theta):
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
    t = torch.arange(max_pos, dtype=torch.float64)
    f = torch.outer(t, inv)
    return torch.cat([f.cos(), f.sin()], dim=-1).float()


def test_rope_qkv_and_kv_copy():
    ops = _ops()
    T, Hq, Hkv, D = 50, 8, 2, 128
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device="cuda", dtype=torch.bfloat16)
    pos = torch.arange(T, device="cuda", dtype=torch.int32) + 7
    cs = _rope_cache(128, D, 500000.0).cuda()
    kd = torch.zeros(T, Hkv, D, device="cuda", dtype=torch.bfloat16)
    vd = torch.zeros_like(kd)
    ref = qkv.float().clone()
    ops.rope_qkv(qkv, Hq, Hkv, D, pos, cs, kd, vd)
    c = cs[pos.long(), : D // 2]
    s = cs[pos.long(), D // 2:]
    for h in range(Hq + Hkv):
        x = ref[:, h * D:(h + 1) * D]
        x1, x2 = x[:, : D // 2], x[:, D // 2:]
        ref[:, h * D:(h + 1) * D] = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)
    assert _rel_err(qkv[:, : (Hq + Hkv) * D], ref[:, : (Hq + Hkv) * D]) < 1e-2
    assert torch.equal(kd.reshape(T, -1), qkv[:, Hq * D:(Hq + Hkv) * D])
    assert torch.equal(vd.reshape(T, -1), qkv[:, (Hq + Hkv) * D:])


def test_silu_mul_embedding_argmax():
    ops = _ops()
    gu = torch.randn(9, 2 * 1024, device="cuda", dtype=torch.bfloat16)
    y = ops.silu_mul(gu)
    g, u = gu.float().chunk(2, -1)
    assert _rel_err(y, torch.nn.functional.silu(g) * u) < 1e-2
    table = torch.randn(1000, 256, device="cuda", dtype=torch.bfloat16)
    ids = torch.randint(0, 1000, (17,), device="cuda", dtype=torch.int32)
    assert torch.equal(ops.embedding(ids, table), table[ids.long()])
    logits = torch.randn(3, 128256, device="cuda", dtype=torch.bfloat16)
    assert torch.equal(ops.argmax(logits).long(), logits.float().argmax(-1))


def _ref_causal(qkv, Hq, Hkv, D=128):
    T = qkv.shape[0]
    q = qkv[:, : Hq * D].float().view(T, Hq, D).transpose(0, 1)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].float().view(T, Hkv, D).transpose(0, 1)
    v = qkv[:, (Hq + Hkv) * D:].float().view(T, Hkv, D).transpose(0, 1)
    g = Hq // Hkv
    k = k.repeat_interleave(g, 0)
    v = v.repeat_interleave(g, 0)
    s = q @ k.transpose(1, 2) / math.sqrt(D)
    mask = torch.ones(T, T, device=qkv.device, dtype=torch.bool).triu(1)
    s.masked_fill_(mask, float("-inf"))
    return (s.softmax(-1) @ v).transpose(0, 1).reshape(T, Hq * D)


@pytest.mark.parametrize("kstages,poly", [(2, 0), (3, 0), (2, 0x11), (2, 0xFF)])
@pytest.mark.parametrize("T,Hq,Hkv", [(128, 1, 1), (200, 4, 2), (1000, 8, 2), (2048, 32, 8)])
def test_flash_prefill(T, Hq, Hkv, kstages, poly):
    ops = _ops()
    torch.manual_seed(1)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * 128, device="cuda", dtype=torch.bfloat16)
    o = ops.flash_prefill(qkv, Hq, Hkv, kstages=kstages, poly=poly)
    ops.check_device_status()
    assert _rel_err(o, _ref_causal(qkv, Hq, Hkv)) < 2e-2


@pytest.mark.parametrize("B,Hq,Hkv,D,ctx", [(1, 32, 8, 128, 8193), (3, 8, 2, 128, 300), (2, 8, 8, 64, 77),
                                             (1, 14, 2, 128, 5000), (2, 28, 4, 128, 700), (1, 24, 8, 128, 333),
                                             (1, 16, 2, 128, 5000), (3, 64, 8, 128, 700)])
def test_paged_decode(B, Hq, Hkv, D, ctx):
    ops = _ops()
    torch.manual_seed(2)
    bs = 16
    nblk_seq = (ctx + bs - 1) // bs
    nb = B * nblk_seq + 3
    kc = torch.randn(nb, bs, Hkv, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    perm = torch.randperm(nb, device="cuda")[: B * nblk_seq].view(B, nblk_seq).to(torch.int32)
    lens = torch.tensor([ctx - i for i in range(B)], device="cuda", dtype=torch.int32)
    q = torch.randn(B, Hq, D, device="cuda", dtype=torch.bfloat16)
    o = ops.paged_decode_attention(q, kc, vc, perm, lens, ctx)
    g = Hq // Hkv
    for b in range(B):
        L = int(lens[b])
        ks = kc[perm[b].long()].reshape(-1, Hkv, D)[:L].float().repeat_interleave(g, 1)
        vs = vc[perm[b].long()].reshape(-1, Hkv, D)[:L].float().repeat_interleave(g, 1)
        s = torch.einsum("hd,thd->ht", q[b].float(), ks) / math.sqrt(D)
        ref = torch.einsum("ht,thd->hd", s.softmax(-1), vs)
        assert _rel_err(o[b], ref) < 1e-2


@pytest.mark.parametrize("n,bits", [(1, 1), (19, 3), (4096, 4), (1000003, 2), (77, 8), (1024, 5)])
def test_bitpack_roundtrip_and_format(n, bits):
    ops = _ops()
    from kvserve_b200.ops.kv_codec import _pack_bits, bitpack_header
    x = torch.randint(0, 2 ** bits, (n,), dtype=torch.uint8)
    out = torch.empty(16 + (n * bits + 7) // 8, dtype=torch.uint8, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.ext().bitpack_encode(x.cuda(), out, bits, st)
    expect = bitpack_header(bits, n) + _pack_bits(x.numpy(), bits)
    assert bytes(out.cpu().numpy().tobytes()) == expect
    back = torch.empty(n, dtype=torch.uint8, device="cuda")
    ops.ext().bitpack_decode(out, back, bits, st)
    assert int(st.item()) == 0
    assert torch.equal(back.cpu(), x)


def test_bitpack_reports_bad_symbol_and_header():
    ops = _ops()
    x = torch.full((64,), 9, dtype=torch.uint8, device="cuda")
    out = torch.empty(16 + 64 * 3 // 8, dtype=torch.uint8, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.ext().bitpack_encode(x, out, 3, st)
    assert int(st.item()) == 3
    st.zero_()
    out[0] ^= 0xFF
    ops.ext().bitpack_decode(out, torch.empty(64, dtype=torch.uint8, device="cuda"), 3, st)
    assert int(st.item()) == 2


@pytest.mark.parametrize("n", [128, 96, 100, 64])
def test_fwht_rows(n):
    ops = _ops()
    from kvserve_b200.ops.kv_codec import hadamard_matrix
    x = torch.randn(33, n, dtype=torch.bfloat16)
    signs = (torch.randint(0, 2, (33, n)) * 2 - 1).float()
    y = torch.empty_like(x.cuda())
    ops.ext().fwht_rows(x.cuda(), y, signs.cuda(), False)
    chunks, rem = [], n
    while rem:
        c = 1 << (rem.bit_length() - 1)
        chunks.append(c)
        rem -= c
    ref = []
    start = 0
    xs = x.float() * signs
    for c in chunks:
        ref.append(xs[:, start:start + c] @ (hadamard_matrix(c) / math.sqrt(c)))
        start += c
    ref = torch.cat(ref, -1)
    assert _rel_err(y.cpu(), ref) < 1e-2


def _codec_case(T, H, D, n_low, kb, vb, raw=False):
    from kvserve_b200.ops import kv_codec as kc
    from kvserve_b200.compression.heads import rademacher_signs, pack_sign_bits
    torch.manual_seed(3)
    k = torch.randn(T, H, D, dtype=torch.bfloat16)
    k[:, :, :4] *= 8  # outlier channels
    v = torch.randn(T, H, D, dtype=torch.bfloat16)
    perm = torch.randperm(H).to(torch.int32)
    spec = kc.spec_from_profile(T, H, D, n_low, (2 ** kb[0], 2 ** kb[1]), (2 ** vb[0], 2 ** vb[1]), raw=raw)
    signs = rademacher_signs(3237919422, 0, H, D)
    return kc, k, v, perm, spec, signs, pack_sign_bits(signs)


@pytest.mark.parametrize("T,H,D,n_low,kb,vb", [(256, 4, 128, 1, (2, 4), (2, 2)), (1000, 8, 128, 3, (3, 4), (2, 4)),
                                               (77, 2, 64, 0, (4, 4), (8, 8)), (33, 8, 256, 8, (4, 4), (2, 2)),
                                               (4096, 8, 128, 6, (4, 4), (2, 2)), (300, 8, 128, 0, (8, 8), (8, 8))])
@pytest.mark.parametrize("allow_mma", [True, False])
def test_kv_codec_matches_cpu_oracle(T, H, D, n_low, kb, vb, allow_mma):
    """head_dim 128 runs the tensor-core encode unless allow_mma is off."""
    kc, k, v, order, spec, signs, sbits = _codec_case(T, H, D, n_low, kb, vb)
    ops = _ops()
    lay = kc.frame_layout(spec)
    assert list(ops.ext().kv_frame_geom(spec.params()))[:2] == [lay.frame_bytes, lay.k_aux]
    frame = torch.zeros(lay.frame_bytes, dtype=torch.uint8, device="cuda")
    state = kc.EncoderState(torch.device("cuda"))
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    kc.encode_layer(k.cuda(), v.cuda(), spec, order.cuda(), sbits.cuda(), frame.data_ptr(), state,
                    flag_ptr=flag.data_ptr(), seq=5, layer=0, allow_mma=allow_mma)
    torch.cuda.synchronize()
    assert int(flag[0].item()) == 5 and int(state.counter[1].item()) == 0
    gpu = frame.cpu().numpy().tobytes()
    cpu = bytes(kc.cpu_encode_frame(k, v, spec, order, signs, layer=0, seq=5))
    assert gpu[:64] == cpu[:64]
    # quantisation parameters (bf16): K per channel, V per token and section
    gk = np.frombuffer(gpu[lay.k_aux:lay.k_aux + 4 * H * D], dtype=np.uint16).astype(np.int32)
    ck = np.frombuffer(cpu[lay.k_aux:lay.k_aux + 4 * H * D], dtype=np.uint16).astype(np.int32)
    assert np.mean(gk != ck) < 2e-2 and np.abs(gk - ck).max() <= 2
    for s in range(2):
        if spec.section_heads(s):
            o = lay.v_aux[s]
            gv = np.frombuffer(gpu[o:o + 4 * T], dtype=np.uint16).astype(np.int32)
            cv = np.frombuffer(cpu[o:o + 4 * T], dtype=np.uint16).astype(np.int32)
            assert np.mean(gv != cv) < 2e-2 and np.abs(gv - cv).max() <= 2
    # symbols: allow a tiny fraction of off-by-one from fp32 summation order
    for p in range(2):
        for s in range(2):
            hs = spec.section_heads(s)
            if hs == 0:
                continue
            off, b = lay.payload[p][s], spec.bits[p][s]
            n = T * hs * D
            assert gpu[off:off + 16] == cpu[off:off + 16]
            g = kc._unpack_bits(gpu[off + 16:off + 16 + (n * b + 7) // 8], b, n).astype(int)
            c = kc._unpack_bits(cpu[off + 16:off + 16 + (n * b + 7) // 8], b, n).astype(int)
            assert np.mean(g != c) < 1e-3 and np.abs(g - c).max() <= 1
    # decode on the GPU into a paged cache and compare with the CPU decoder
    bs = 16
    nblk = (T + bs - 1) // bs
    cache = torch.zeros(1, 2, nblk + 2, bs, H, D, dtype=torch.bfloat16, device="cuda")
    table = (torch.randperm(nblk + 2)[:nblk]).to(torch.int32).cuda()
    st = torch.zeros(4, dtype=torch.int32, device="cuda")
    kc.decode_layers(frame.data_ptr(), lay.frame_bytes, spec, order.view(1, H).cuda(),
                     sbits.view(1, H, D // 32).cuda(), cache, table, st, flags_ptr=flag.data_ptr(), seq=5)
    torch.cuda.synchronize()
    assert int(st[0].item()) == 0
    kd, vd = kc.cpu_decode_frame(cpu, spec, order, signs)
    got = cache[0][:, table.long()].reshape(2, -1, H, D)[:, :T].cpu()
    assert _rel_err(got[0], kd) < 2e-2 and _rel_err(got[1], vd) < 2e-2
    # reconstruction quality vs the original
    assert _rel_err(got[0], k) < 0.35 and _rel_err(got[1], v) < 0.7


def test_kv_codec_raw_sections_exact():
    kc, k, v, order, spec, signs, sbits = _codec_case(100, 4, 128, 2, (4, 4), (4, 4), raw=True)
    lay = kc.frame_layout(spec)
    frame = torch.zeros(lay.frame_bytes, dtype=torch.uint8, device="cuda")
    state = kc.EncoderState(torch.device("cuda"))
    kc.encode_layer(k.cuda(), v.cuda(), spec, order.cuda(), sbits.cuda(), frame.data_ptr(), state, seq=1)
    cache = torch.zeros(1, 2, 7, 16, 4, 128, dtype=torch.bfloat16, device="cuda")
    table = torch.arange(7, dtype=torch.int32, device="cuda")
    st = torch.zeros(4, dtype=torch.int32, device="cuda")
    kc.decode_layers(frame.data_ptr(), lay.frame_bytes, spec, order.view(1, 4).cuda(),
                     sbits.view(1, 4, 4).cuda(), cache, table, st, seq=1)
    got = cache[0].reshape(2, -1, 4, 128)[:, :100].cpu()
    assert torch.equal(got[0], k) and torch.equal(got[1], v)


def test_decode_wait_times_out_without_fault():
    """A flag that nothing publishes: the bounded wait returns a status."""
    kc, k, v, order, spec, signs, sbits = _codec_case(32, 2, 128, 1, (4, 4), (2, 2))
    lay = kc.frame_layout(spec)
    frame = torch.zeros(lay.frame_bytes, dtype=torch.uint8, device="cuda")
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    cache = torch.zeros(1, 2, 2, 16, 2, 128, dtype=torch.bfloat16, device="cuda")
    table = torch.arange(2, dtype=torch.int32, device="cuda")
    st = torch.zeros(4, dtype=torch.int32, device="cuda")
    kc.decode_layers(frame.data_ptr(), lay.frame_bytes, spec, order.view(1, 2).cuda(), sbits.view(1, 2, 4).cuda(),
                     cache, table, st, flags_ptr=flag.data_ptr(), seq=9, timeout_ns=50_000_000)
    torch.cuda.synchronize()
    assert int(st[0].item()) == 1
    # the context is still usable
    assert float(torch.ones(4, device="cuda").sum().item()) == 4.0


@pytest.mark.parametrize("n", [5, 16384, 100000, 3 * 16384 + 17])
def test_lossless_gpu_matches_cpu_bytes(n):
    from kvserve_b200.compression.codec.lossless import encode_bytes, decode_bytes
    from kvserve_b200.ops.lossless import gpu_encode, gpu_decode
    g = torch.Generator().manual_seed(n)
    x = torch.randint(0, 16, (n,), generator=g, dtype=torch.uint8)
    x[: n // 4] = 0
    if n > 50000:
        x[50000:60000] = torch.randint(0, 256, (10000,), generator=g, dtype=torch.uint8)  # incompressible chunk
    enc = gpu_encode(x.cuda())
    ref = encode_bytes(x.numpy())
    assert bytes(enc.cpu().numpy().tobytes()) == ref
    back = gpu_decode(enc)
    assert torch.equal(back.cpu(), x)
    assert torch.equal(torch.from_numpy(decode_bytes(ref)), x)


@pytest.mark.parametrize("T", [255, 511, 1023, 4095])
def test_flash_prefill_partial_tiles_llama_heads(T):
    """Prompt lengths T-1 of power-of-two prompts (the engine's prefill sizes)."""
    ops = _ops()
    torch.manual_seed(T)
    qkv = torch.randn(T, (32 + 16) * 128, device="cuda", dtype=torch.bfloat16) * 2.0
    o = ops.flash_prefill(qkv, 32, 8)
    ops.check_device_status()
    assert _rel_err(o, _ref_causal(qkv, 32, 8)) < 2e-2


@pytest.mark.parametrize("Ms,N,K", [((300, 1024, 129), 1024, 512), ((8192,), 4096, 2048)])
def test_gemm_allreduce_single_rank(Ms, N, K):
    """Mode-3 epilogue with one rank: every tile is owned locally and leaves
    through the shared-memory slab; successive launches advance the epoch."""
    ops = _ops()
    from kvserve_b200.parallel.tp_allreduce import TPAllReduce
    ws = TPAllReduce(1, 0, max(Ms), N, torch.device("cuda", 0))
    ws.connect([None])
    try:
        torch.manual_seed(1)
        b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
        for M in Ms:
            a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
            c = ws.gemm_allreduce(a, b).clone()
            ops.check_device_status()
            ref = a.float() @ b.float().T
            assert _rel_err(c, ref) < 1e-2
            assert torch.equal(c, ops.gemm(a, b))   # same fp32 tile, one rounding
    finally:
        ws.close()


@pytest.mark.parametrize("mean_dtype,refine,group,kb,vb", [("float32", 1, 128, 3, 2), ("bfloat16", 2, 32, 4, 1),
                                                           ("float32", 0, 16, 2, 4)])
def test_centered_codebook_cuda_matches_cpu(mean_dtype, refine, group, kb, vb):
    from kvserve_b200.compression.quantizer.centered_codebook import CenteredCodebookQuantizer
    torch.manual_seed(0)
    kv = torch.randn(2, 5, 16, 4, 128, dtype=torch.bfloat16)   # 80 tokens: a partial last key group
    kv[0, ..., :4] *= 8
    qz = CenteredCodebookQuantizer(key_bits=kb, value_bits=vb, group_size=group, scale_refinements=refine,
                                   mean_dtype=mean_dtype)
    q_cpu, m_cpu = qz.quantize(0, kv)
    q_gpu, m_gpu = qz.quantize(0, kv.cuda())
    assert (q_gpu.cpu() == q_cpu).float().mean().item() > 0.999
    for pc, pg in zip(m_cpu["parts"], m_gpu["parts"]):
        assert pg["mean"].dtype == pc["mean"].dtype and pg["scale"].shape == pc["scale"].shape
        torch.testing.assert_close(pg["scale"].cpu().float(), pc["scale"].float(), rtol=1e-2, atol=1e-3)
        torch.testing.assert_close(pg["mean"].cpu().float(), pc["mean"].float(), rtol=1e-2, atol=1e-3)
    # identical symbols and parameters dequantise to identical values
    m_on_gpu = dict(m_cpu, parts=[{k: v.cuda() for k, v in p.items()} for p in m_cpu["parts"]])
    assert torch.equal(qz.dequantize(0, q_cpu.cuda(), m_on_gpu).cpu(), qz.dequantize(0, q_cpu, m_cpu))
    err = lambda r: ((r.float().cpu() - kv.float()).norm() / kv.float().norm()).item()  # noqa: E731
    assert abs(err(qz.dequantize(0, q_gpu, m_gpu)) - err(qz.dequantize(0, q_cpu, m_cpu))) < 1e-3
    bad = q_gpu.clone()
    bad[1, 0, 0, 0, 0] = 1 << vb
    with pytest.raises(ValueError):
        qz.dequantize(0, bad, m_gpu)


@pytest.mark.parametrize("M", [1, 3, 8])
def test_fused_lm_head_argmax_matches_unfused(M):
    """LM-head GEMV + greedy argmax in one launch (one rank) picks the token
    of the bf16 logits of the separate GEMV, ties to the smallest index."""
    from kvserve_b200 import ops
    from kvserve_b200.parallel.context import ParallelContext
    from kvserve_b200.parallel.decode_allreduce import create_decode_collectives
    V, K = 128256 // 8, 4096
    dc = create_decode_collectives(ParallelContext(), K, V, num_sites=1, device=torch.device("cuda"))
    g = torch.Generator(device="cuda").manual_seed(M)
    for rep in range(2):   # the completion counter resets itself
        h = torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g)
        head = torch.randn(V, K, device="cuda", dtype=torch.bfloat16, generator=g) * 0.02
        tok = dc.greedy(h, head, 0, site=0)
        ref = ops.argmax(ops.linear(h, head))
        torch.cuda.synchronize()
        assert torch.equal(tok, ref)
    dc.close()
