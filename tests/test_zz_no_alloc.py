"""The allocation-free C entry point of paged decode attention.

It exists for callers that cannot allocate device memory when they launch
work (a pool handed entirely to the KV cache, code inside an allocator hook,
a C host program without PyTorch).  This test calls it through its exported
C symbol — exactly as such a caller would — and checks it against the
regular entry point on two calls in a row, so results cannot depend on what
an earlier call left in the shared scratch array.  The file name sorts last
so that a run which stops at the first failure has run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import kvserve_b200._C as ext_mod
    lib = ctypes.CDLL(ext_mod.__file__)
    f = lib.kvs_paged_decode_attention_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                  ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p,
                  ctypes.c_int64, ctypes.c_void_p]
    lib.kvs_noalloc_error_string.restype = ctypes.c_char_p
    lib.kvs_noalloc_error_string.argtypes = [ctypes.c_int]
    lib.kvs_paged_decode_noalloc_capacity.restype = ctypes.c_int64
    return lib


def _rel_err(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _case(seed, B, Hq, Hkv, D, ctx, bs=16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    nblk = (ctx + bs - 1) // bs
    nb = B * nblk + 5
    k = torch.randn(nb, bs, Hkv, D, generator=g).to(torch.bfloat16).cuda()
    v = torch.randn(nb, bs, Hkv, D, generator=g).to(torch.bfloat16).cuda()
    table = torch.randperm(nb, generator=g)[: B * nblk].view(B, nblk).to(torch.int32).cuda()
    lens = torch.tensor([max(1, ctx - 7 * i) for i in range(B)], dtype=torch.int32).cuda()
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16).cuda()
    return q, k, v, table, lens


def _call(lib, q, k, v, table, lens, ctx, out):
    B, Hq, D = q.shape
    Hkv = k.shape[2]
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.kvs_paged_decode_attention_noalloc(
        q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
        table.data_ptr(), table.stride(0), lens.data_ptr(), B, Hq, Hkv, D, k.shape[1], ctx, D ** -0.5,
        out.data_ptr(), out.stride(0), stream)
    return rc


@pytest.mark.parametrize("B,Hq,Hkv,D,ctx", [(1, 32, 8, 128, 8193), (3, 8, 2, 128, 1000), (2, 8, 8, 64, 300)])
def test_noalloc_matches_regular_entry_point_twice(B, Hq, Hkv, D, ctx):
    from kvserve_b200 import ops
    lib = _lib()
    for call in range(2):  # two calls in a row, different inputs, shared scratch
        q, k, v, table, lens = _case(100 * call + B, B, Hq, Hkv, D, ctx)
        ref = ops.paged_decode_attention(q, k, v, table, lens, ctx)
        out = torch.empty_like(q)
        rc = _call(lib, q, k, v, table, lens, ctx, out)
        assert rc == 0, lib.kvs_noalloc_error_string(rc).decode()
        torch.cuda.synchronize()
        assert _rel_err(out, ref) < 1e-2


def test_noalloc_rejects_oversized_schedule():
    lib = _lib()
    cap = lib.kvs_paged_decode_noalloc_capacity()
    assert cap == 2048
    # 37 sequences x 8 query heads x 8 splits = 2368 partial records > 2048
    B, Hq, Hkv, D, ctx = 37, 8, 1, 128, 4096
    q = torch.zeros(B, Hq, D, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(4, 16, Hkv, D, dtype=torch.bfloat16, device="cuda")
    table = torch.zeros(B, 1, dtype=torch.int32, device="cuda")
    lens = torch.ones(B, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    rc = _call(lib, q, k, k, table, lens, ctx, out)
    assert rc == 2 and b"2048" in lib.kvs_noalloc_error_string(rc)
