"""GPU: moe_align_noalloc, the align stage for callers that cannot allocate device memory.

Some callers cannot give this library a scratch buffer: their device memory is
owned by a host engine that reserves it up front and allows no side
allocations, or they reach the library through a foreign-function binding with
no access to that engine's allocator. moe_align_noalloc serves them with a
fixed scratch array inside the library. This test calls it through the C ABI
twice in a row (different inputs, so the second call must not see the first
call's scratch contents) and checks each result against the allocating entry
point moe_align on the same input: counts and block_start exactly, each
expert's rows as the same set of pair ids, padding rows -1.

The file name sorts last so that a run stopping at the first failure has run
every other test before this one.
"""
import ctypes

import numpy as np
import pytest
import torch

from kernelswift_competition_submission_b200 import _lib, moe_align

pytestmark = pytest.mark.gpu


def _noalloc(ids: torch.Tensor, E: int, bm: int):
    lib = _lib.load()
    flat = ids.to(torch.int32).contiguous().view(-1)
    P = flat.numel()
    cap = lib.moe_align_capacity(P, E, bm)
    dev = ids.device
    counts = torch.full((E,), -7, dtype=torch.int32, device=dev)
    bs = torch.full((E + 1,), -7, dtype=torch.int32, device=dev)
    sp = torch.full((max(cap, 1),), -7, dtype=torch.int32, device=dev)
    rc = lib.moe_align_noalloc(flat.data_ptr(), P, E, bm, counts.data_ptr(), bs.data_ptr(), sp.data_ptr(), cap,
                               torch.cuda.current_stream(dev).cuda_stream)
    assert rc == _lib.MOE_OK, _lib.status_string(rc)
    return counts, bs, sp[:cap]


def _same(a, b, bm):
    ca, ba, sa = (t.cpu().numpy() for t in a)
    cb, bb, sb = (t.cpu().numpy() for t in b)
    np.testing.assert_array_equal(ca, cb)
    np.testing.assert_array_equal(ba, bb)
    for e in range(len(ca)):
        r0, r1 = int(ba[e]) * bm, int(ba[e + 1]) * bm
        np.testing.assert_array_equal(np.sort(sa[r0:r1]), np.sort(sb[r0:r1]))
        assert (sa[r0 + ca[e]:r1] == -1).all()


def test_noalloc_align_matches_allocating_entry_point(cuda_device):
    gen = torch.Generator(device=cuda_device).manual_seed(11)
    first = torch.randint(0, 256, (4096, 8), generator=gen, device=cuda_device, dtype=torch.int32)
    second = torch.randint(0, 64, (777, 6), generator=gen, device=cuda_device, dtype=torch.int32)
    for ids, E in ((first, 256), (second, 64)):
        got = _noalloc(ids, E, 128)
        ref = moe_align(ids, E, 128)
        torch.cuda.synchronize()
        _same(got, ref, 128)


def test_noalloc_align_rejects_oversized_request(cuda_device):
    lib = _lib.load()
    p = ctypes.c_void_p(256)
    rc = lib.moe_align_noalloc(p, 8, _lib.MOE_NOALLOC_MAX_EXPERTS + 1, 128, p, p, p, 1 << 20, None)
    assert rc == _lib.MOE_ERR_SCRATCH_LIMIT
    assert "scratch" in _lib.status_string(rc)
