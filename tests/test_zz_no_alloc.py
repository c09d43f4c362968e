"""The allocation-free FFN entry point, called through the C ABI.

tjb_ffn_noalloc exists for callers that cannot allocate device memory when
they call in (a fixed memory pool with no allocator hook, or a path where an
allocation may not block or fail): it keeps the FFN's hidden activations in a
fixed 16 MiB array inside the library instead of caller scratch.  It runs the
same two GEMMs on the same inputs as tjb_ffn, which takes that scratch from
the caller, so its output must be bit-identical -- on the first call and on a
second call, when the shared array still holds the first call's contents.
This file is collected last on purpose.
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ffn_pair(t, d, f, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    h = torch.randn(t, d, device="cuda", generator=g).half()
    w1 = (torch.randn(f, d, device="cuda", generator=g) / math.sqrt(d)).half()
    w2 = (torch.randn(d, f, device="cuda", generator=g) / math.sqrt(f)).half()
    b1 = torch.randn(f, device="cuda", generator=g)
    b2 = torch.randn(d, device="cuda", generator=g)
    return h, w1, b1, w2, b2


def test_noalloc_matches_ffn_twice():
    from tjkernels import _lib
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    # Two calls in a row with different inputs and shapes: the second runs
    # on the array the first one left behind.
    for t, d, f, seed in ((1000, 1024, 4096, 11), (512, 768, 3072, 12)):
        h, w1, b1, w2, b2 = _ffn_pair(t, d, f, seed)
        ref = torch.empty(t, d, dtype=torch.float32, device="cuda")
        hidden = torch.empty(t, f, dtype=torch.float16, device="cuda")
        _lib.check(lib.tjb_ffn(h.data_ptr(), w1.data_ptr(), b1.data_ptr(), w2.data_ptr(),
                               b2.data_ptr(), ref.data_ptr(), hidden.data_ptr(), t, d, f,
                               _lib.TJB_F16, _lib.TJB_F32, stream), "tjb_ffn")
        got = torch.full((t, d), float("nan"), dtype=torch.float32, device="cuda")
        _lib.check(lib.tjb_ffn_noalloc(h.data_ptr(), w1.data_ptr(), b1.data_ptr(),
                                       w2.data_ptr(), b2.data_ptr(), got.data_ptr(), t, d, f,
                                       _lib.TJB_F16, _lib.TJB_F32, stream), "tjb_ffn_noalloc")
        torch.cuda.synchronize()
        # Same kernels, same operands, same order of summation: bit-identical.
        assert torch.equal(got, ref)


def test_noalloc_rejects_oversize():
    """T * F one past the array's limit is refused before anything launches.
    Every buffer is as large as the shape claims, so even a regressed guard
    could not read or write outside them."""
    from tjkernels import _lib
    lib = _lib.lib()
    d, f = 64, 64
    t = (8 << 20) // f + 1  # T * F just over the 8 Mi-element limit
    h, w1, b1, w2, b2 = _ffn_pair(t, d, f, 3)
    out = torch.zeros(t, d, device="cuda")
    status = lib.tjb_ffn_noalloc(h.data_ptr(), w1.data_ptr(), b1.data_ptr(), w2.data_ptr(),
                                 b2.data_ptr(), out.data_ptr(), t, d, f,
                                 _lib.TJB_F16, _lib.TJB_F32,
                                 torch.cuda.current_stream().cuda_stream)
    assert status == 2  # TJB_ERR_BAD_SHAPE, nothing launched
    torch.cuda.synchronize()
    assert (out == 0).all()
