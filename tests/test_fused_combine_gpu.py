"""The top-k combine fused into the down GEMM's epilogue gives the bits of the separate combine.

Both endings of the expert path run on the same workspace after the same align and gate/up
GEMM stages, through the C ABI: ``moe_expert_gemm2`` + ``moe_expert_combine`` (slot rows, then
a weighted sum per token) against ``moe_expert_gemm2_combine`` (the warp that stores a token's
last slot of an n-block sums that token's slots). The fused sum runs in slot order in fp32 with
one rounding, as the separate combine does, so the outputs are compared bit for bit. The cases
cover the down GEMM's two tile widths (K < 256 and K >= 256, ragged last n-block), top-k above
one load batch of 8, slots whose expert id is outside [0, E), and tokens with no valid slot at
all (their rows must come out as zeros, as in the reference's expert loop,
fused_moe/v0/fused_moe.py:154-167).
"""
import pytest
import torch

from kernelswift_competition_submission_b200 import _lib, check_device_status
from kernelswift_competition_submission_b200.ops import _DTYPES, _ptr, _stream, status_word
from torch_ref import experts_rows_fp32

pytestmark = pytest.mark.gpu


def _case(M, E, k, K, N, dev, seed, dtype=torch.bfloat16):
    gen = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, K, generator=gen, device=dev).to(dtype)
    w1 = (torch.randn(E, 2 * N, K, generator=gen, device=dev) / K ** 0.5).to(dtype)
    w2 = (torch.randn(E, K, N, generator=gen, device=dev) / N ** 0.5).to(dtype)
    ids = torch.randint(0, E, (M, k), generator=gen, device=dev, dtype=torch.int32)
    w = torch.rand(M, k, generator=gen, device=dev)
    if M > 3:
        ids[1::3, -1] = -1       # a skipped slot
        ids[2::7, 0] = E + 5     # an id outside [0, E): contributes nothing
        ids[3::11, :] = -1       # tokens with no valid slot
    return x, w1, w2, w, ids


@pytest.mark.parametrize("M,E,k,K,N", [(1, 8, 2, 256, 128), (83, 8, 2, 128, 64), (300, 16, 4, 512, 256),
                                       (1000, 32, 8, 1024, 320), (129, 4, 1, 192, 192), (64, 8, 12, 320, 128),
                                       (2048, 16, 8, 2048, 512)])
def test_fused_combine_same_bits(cuda_device, M, E, k, K, N):
    dev = cuda_device
    x, w1, w2, w, ids = _case(M, E, k, K, N, dev, seed=M * 7 + K)
    lib = _lib.load()
    dt = _DTYPES[x.dtype]
    need = int(lib.moe_fused_workspace_bytes(M, E, k, K, N))
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    st, status = _stream(dev), _ptr(status_word(dev))
    _lib.check(lib.moe_expert_align_gather(dt, _ptr(x), _ptr(ids), M, E, k, K, N, _ptr(ws), need, st), "align")
    _lib.check(lib.moe_expert_gemm1(dt, _ptr(w1), M, E, k, K, N, _ptr(ws), need, status, 0, st), "gemm1")
    sep = torch.full((M, K), float("nan"), dtype=x.dtype, device=dev)
    _lib.check(lib.moe_expert_gemm2(dt, _ptr(w2), M, E, k, K, N, _ptr(ws), need, status, 0, st), "gemm2")
    _lib.check(lib.moe_expert_combine(dt, _ptr(w), _ptr(ids), M, E, k, K, N, _ptr(sep), _ptr(ws), need, st),
               "combine")
    fused = torch.full((M, K), float("nan"), dtype=x.dtype, device=dev)
    for _ in range(2):  # a second call reuses the workspace: the arrival counters start from zero again
        _lib.check(lib.moe_expert_gemm2_combine(dt, _ptr(w2), _ptr(w), _ptr(ids), M, E, k, K, N, _ptr(fused),
                                                _ptr(ws), need, status, 0, st), "gemm2_combine")
        torch.cuda.synchronize()
        check_device_status(dev)
        assert torch.equal(fused, sep)
    # and the whole single-call entry point
    one = torch.full((M, K), float("nan"), dtype=x.dtype, device=dev)
    _lib.check(lib.moe_fused_experts(dt, _ptr(x), _ptr(w1), _ptr(w2), _ptr(w), _ptr(ids), M, E, k, K, N, _ptr(one),
                                     _ptr(ws), need, status, st), "fused_experts")
    torch.cuda.synchronize()
    assert torch.equal(one, sep)
    empty = (((ids < 0) | (ids >= E)).all(dim=1)).nonzero().flatten()
    if empty.numel():
        assert torch.count_nonzero(one[empty]) == 0
    rows = torch.arange(0, M, max(1, M // 64))
    ref = experts_rows_fp32(x, w1, w2, w * ((ids >= 0) & (ids < E)), ids.clamp(0, E - 1), rows)
    torch.testing.assert_close(one[rows.to(dev)].float(), ref, atol=2e-2, rtol=2e-2)


def test_fused_combine_fp16(cuda_device):
    dev = cuda_device
    M, E, k, K, N = 257, 8, 2, 384, 192
    x, w1, w2, w, ids = _case(M, E, k, K, N, dev, seed=5, dtype=torch.float16)
    from kernelswift_competition_submission_b200 import fused_moe

    out = fused_moe(x, w1, w2, w, ids)
    rows = torch.arange(0, M, 3)
    ref = experts_rows_fp32(x, w1, w2, w * ((ids >= 0) & (ids < E)), ids.clamp(0, E - 1), rows)
    torch.testing.assert_close(out[rows.to(dev)].float(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("M,E,k,K,N", [(1, 8, 2, 256, 128), (83, 8, 2, 128, 64), (300, 16, 4, 512, 256),
                                       (1000, 32, 8, 1024, 320), (129, 4, 1, 192, 192), (2048, 16, 8, 2048, 512)])
def test_gemm1_row_gather_same_bits(cuda_device, M, E, k, K, N):
    """The gate/up GEMM reading its A rows straight from the token rows (cp.async into the
    swizzled tile) gives the bits of the GEMM on the expert-sorted copy of the rows."""
    dev = cuda_device
    x, w1, w2, w, ids = _case(M, E, k, K, N, dev, seed=M + 3 * K)
    lib = _lib.load()
    dt = _DTYPES[x.dtype]
    need = int(lib.moe_fused_workspace_bytes(M, E, k, K, N))
    st, status = _stream(dev), _ptr(status_word(dev))
    outs = []
    for gather_in_gemm in (False, True):
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        out = torch.full((M, K), float("nan"), dtype=x.dtype, device=dev)
        if gather_in_gemm:
            _lib.check(lib.moe_expert_align(_ptr(ids), M, E, k, K, N, _ptr(ws), need, st), "align")
            _lib.check(lib.moe_expert_gemm1_gather(dt, _ptr(x), _ptr(w1), M, E, k, K, N, _ptr(ws), need, status, 0,
                                                   st), "gemm1_gather")
        else:
            _lib.check(lib.moe_expert_align_gather(dt, _ptr(x), _ptr(ids), M, E, k, K, N, _ptr(ws), need, st),
                       "align_gather")
            _lib.check(lib.moe_expert_gemm1(dt, _ptr(w1), M, E, k, K, N, _ptr(ws), need, status, 0, st), "gemm1")
        _lib.check(lib.moe_expert_gemm2(dt, _ptr(w2), M, E, k, K, N, _ptr(ws), need, status, 0, st), "gemm2")
        _lib.check(lib.moe_expert_combine(dt, _ptr(w), _ptr(ids), M, E, k, K, N, _ptr(out), _ptr(ws), need, st),
                   "combine")
        torch.cuda.synchronize()
        check_device_status(dev)
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
