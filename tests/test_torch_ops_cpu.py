"""CPU: the torch.library registrations (torch.ops.moe_b200.*) and their fake
implementations, which give output shapes and dtypes without running a kernel."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import kernelswift_competition_submission_b200  # noqa: F401  (registers the operators)


def test_operators_registered():
    for name in ("grouped_topk", "fused_moe", "fused_moe_fp8", "moe_align", "quantize_rows_fp8",
                 "quantize_weights_fp8"):
        assert hasattr(torch.ops.moe_b200, name), name


def test_fake_shapes():
    with FakeTensorMode():
        x = torch.empty(37, 512, dtype=torch.bfloat16)
        g = torch.empty(37, 16)
        w, ids = torch.ops.moe_b200.grouped_topk(x, g, 4, True, 4, 2, "sigmoid", 2.5, torch.empty(16))
        assert w.shape == (37, 4) and w.dtype == torch.float32 and ids.dtype == torch.int32
        w1 = torch.empty(16, 512, 512, dtype=torch.bfloat16)
        w2 = torch.empty(16, 512, 256, dtype=torch.bfloat16)
        out = torch.ops.moe_b200.fused_moe(x, w1, w2, w, ids)
        assert out.shape == x.shape and out.dtype == x.dtype
        q, s = torch.ops.moe_b200.quantize_rows_fp8(x)
        assert q.dtype == torch.float8_e4m3fn and s.shape == (37, 4)
        w1q, w1s = torch.ops.moe_b200.quantize_weights_fp8(w1)
        w2q, w2s = torch.ops.moe_b200.quantize_weights_fp8(w2)
        assert w1s.shape == (16, 4, 4) and w2s.shape == (16, 4, 2)
        o8 = torch.ops.moe_b200.fused_moe_fp8(x, w1q, w1s, w2q, w2s, w, ids)
        assert o8.shape == x.shape and o8.dtype == torch.bfloat16
        counts, block_start, pairs = torch.ops.moe_b200.moe_align(ids, 16, 128)
        assert counts.shape == (16,) and block_start.shape == (17,)
        assert pairs.shape == ((37 * 4 + 16 * 127 + 127) // 128 * 128,)


def test_weights_scale_format_follows_tensor_not_address():
    """The power-of-two check is remembered on each scale tensor with its _version: an in-place
    change is seen, and a new tensor (even at a reused address) is checked afresh."""
    from kernelswift_competition_submission_b200 import weights_scale_format

    a = torch.full((2, 4, 3), 0.25)
    assert weights_scale_format(a, a) == "ue8m0"
    a.mul_(1.5)
    assert weights_scale_format(a, a) == "fp32"
    for _ in range(20):  # fresh tensors, which the allocator may place where freed ones were
        b = torch.full((2, 4, 3), 0.3)
        assert weights_scale_format(b, b) == "fp32"
        del b
        c = torch.full((2, 4, 3), 0.125)
        assert weights_scale_format(c, c) == "ue8m0"
        del c
