"""BitPack payloads byte-identical with the reference's own GPU codec.

The reference packs with a Triton kernel (kvserve_v1/compression/codec/bitpack_codec.py:25-135);
this framework packs with its sm_100a ``bitpack_encode`` kernel.  For every
width 1-8 and several lengths (including ones whose packed size is not a
whole word) the two payloads must be the same bytes, and each side must
decode the other's payload to the original symbols.
"""
import os
import sys

import pytest
import torch

from kvserve_b200.baselines.reference_arm import REF_DIR

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not os.path.isdir(os.path.join(REF_DIR, "kvserve_v1")),
                                 reason="reference not installed in baseline/_ref")]


@pytest.mark.parametrize("bits", range(1, 9))
@pytest.mark.parametrize("n", [1, 7, 1000, 65537])
def test_bitpack_bytes_equal_reference(bits, n):
    sys.path.insert(0, REF_DIR)
    try:
        from kvserve_v1.compression.codec.bitpack_codec import BitPackCodec as RefCodec
    finally:
        sys.path.remove(REF_DIR)
    from kvserve_b200.compression.codec.bitpack import BitPackCodec
    g = torch.Generator().manual_seed(bits * 100003 + n)
    sym = torch.randint(0, 1 << bits, (n,), generator=g, dtype=torch.uint8).cuda()
    ref, ours = RefCodec(bitpack_bits=bits), BitPackCodec(bitpack_bits=bits)
    a = ref.encode(sym)
    b = ours.encode(sym)
    torch.cuda.synchronize()
    assert torch.equal(a.cpu(), b.cpu())
    assert torch.equal(ours.decode(a, "uint8", [n], "cuda"), sym)
    assert torch.equal(ref.decode(b, "uint8", [n], "cuda"), sym)
