"""The allocation-free C entry point of paged decode attention.

It exists for callers that cannot allocate device memory when they launch
work (a pool handed entirely to the KV cache, code inside an allocator hook,
a C host program without PyTorch).  This test calls it through its exported
C symbol, exactly as such a caller would, with the argument types read from
its C header ``csrc/paged_decode_noalloc.h`` (so the test follows the
declared interface), and checks it against the regular entry point on two
calls in a row, so results cannot depend on what an earlier call left in the
shared scratch array.  The file name sorts last so that a run which stops at
the first failure has run every other test.
"""
import ctypes
import os
import re

import pytest
import torch

pytestmark = pytest.mark.gpu

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "csrc", "paged_decode_noalloc.h")

_CTYPES = {"int": ctypes.c_int, "int64_t": ctypes.c_int64, "float": ctypes.c_float}


def _header_prototypes() -> dict:
    """name -> (restype, argtypes) of every function the header declares."""
    text = re.sub(r"//[^\n]*", "", open(HEADER).read())
    out = {}
    for ret, name, args in re.findall(r"([\w\s\*]+?)\s*\b(kvs_\w+)\s*\(([^)]*)\)\s*;", text):
        def ct(decl: str):
            decl = decl.strip()
            if "*" in decl:
                return ctypes.c_char_p if decl.startswith("const char") else ctypes.c_void_p
            return _CTYPES[decl.replace("const", "").split()[0]]
        params = [a for a in args.split(",") if a.strip() and a.strip() != "void"]
        # drop the parameter name, keep its type
        types = [ct(re.sub(r"\b\w+\s*$", "", p)) for p in params]
        out[name] = (ct(ret.split("\n")[-1]), types)
    return out


def _lib():
    import kvserve_b200._C as ext_mod
    lib = ctypes.CDLL(ext_mod.__file__)
    protos = _header_prototypes()
    assert {"kvs_paged_decode_attention_noalloc", "kvs_noalloc_error_string", "kvs_paged_decode_noalloc_capacity",
            "kvs_noalloc_last_cuda_error"} <= set(protos)
    for name, (res, args) in protos.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
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


def _call(lib, q, k, v, table, lens, ctx, out, q_ptr=None):
    B, Hq, D = q.shape
    Hkv = k.shape[2]
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.kvs_paged_decode_attention_noalloc(
        q.data_ptr() if q_ptr is None else q_ptr, q.stride(0), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1),
        k.stride(2), table.data_ptr(), table.stride(0), lens.data_ptr(), B, Hq, Hkv, D, k.shape[1], ctx, D ** -0.5,
        out.data_ptr(), out.stride(0), stream)
    return rc


# (B, Hq, Hkv, D, ctx): long context with 32 splits, 3 sequences, head_dim 64,
# 8 query heads per KV head (G=8), and a short context whose single split
# writes the output directly without touching the scratch array.
@pytest.mark.parametrize("B,Hq,Hkv,D,ctx", [(1, 32, 8, 128, 8193), (3, 8, 2, 128, 1000), (2, 8, 8, 64, 300),
                                            (2, 32, 4, 128, 2048), (2, 32, 8, 128, 100)])
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
    # 37 sequences, 1 KV head, 4096 tokens: min(3 * 148 / 37, 4096 / 128) = 12
    # splits, so 37 x 8 query heads x 12 = 3552 partial records > 2048
    B, Hq, Hkv, D, ctx = 37, 8, 1, 128, 4096
    q = torch.zeros(B, Hq, D, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(4, 16, Hkv, D, dtype=torch.bfloat16, device="cuda")
    table = torch.zeros(B, 1, dtype=torch.int32, device="cuda")
    lens = torch.ones(B, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    rc = _call(lib, q, k, k, table, lens, ctx, out)
    assert rc == 2 and b"2048" in lib.kvs_noalloc_error_string(rc)


def test_noalloc_rejects_misaligned_pointer_without_launching():
    lib = _lib()
    B, Hq, Hkv, D, ctx = 1, 8, 2, 128, 256
    q, k, v, table, lens = _case(7, B, Hq, Hkv, D, ctx)
    out = torch.full_like(q, 3.0)
    torch.cuda.synchronize()
    # 2 bytes past a 16-byte boundary: the vector loads would fault, so the
    # call must refuse before launching anything
    rc = _call(lib, q, k, v, table, lens, ctx, out, q_ptr=q.data_ptr() + 2)
    assert rc == 1, lib.kvs_noalloc_error_string(rc).decode()
    torch.cuda.synchronize()
    assert torch.all(out == 3.0)
    assert lib.kvs_noalloc_last_cuda_error() == 0
