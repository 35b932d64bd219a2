"""GPU: torch.ops.moe_b200.* run the same kernels as the functional API (same bits), pass
torch.library.opcheck (schema, fake implementation, no aliasing of inputs), and trace into
a torch.compile graph without a break. Also the FP8 ModelNew drop-in: its output against the
FP8 expert path, and its quantised-weight cache keyed on the parameters' _version."""
import pytest
import torch

import kernelswift_competition_submission_b200 as pkg

pytestmark = pytest.mark.gpu


def _case(dev, M=64, E=16, K=256, N=128, k=4):
    gen = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(M, K, generator=gen, device=dev).to(torch.bfloat16)
    g = torch.randn(M, E, generator=gen, device=dev)
    bias = torch.randn(E, generator=gen, device=dev) * 0.01
    w1 = (torch.randn(E, 2 * N, K, generator=gen, device=dev) / K ** 0.5).to(torch.bfloat16)
    w2 = (torch.randn(E, K, N, generator=gen, device=dev) / N ** 0.5).to(torch.bfloat16)
    return x, g, bias, w1, w2


def test_ops_same_bits_as_functional(cuda_device):
    x, g, bias, w1, w2 = _case(cuda_device)
    w, ids = torch.ops.moe_b200.grouped_topk(x, g, 4, True, 4, 2, "sigmoid", 2.5, bias)
    w_ref, ids_ref = pkg.grouped_topk(x, g, 4, True, 4, 2, "sigmoid", 2.5, e_score_correction_bias=bias)
    assert torch.equal(w, w_ref) and torch.equal(ids, ids_ref)
    out = torch.ops.moe_b200.fused_moe(x, w1, w2, w, ids)
    assert torch.equal(out, pkg.fused_moe(x, w1, w2, w, ids))
    w1q, w1s = torch.ops.moe_b200.quantize_weights_fp8(w1)
    w2q, w2s = torch.ops.moe_b200.quantize_weights_fp8(w2)
    o8 = torch.ops.moe_b200.fused_moe_fp8(x, w1q, w1s, w2q, w2s, w, ids)
    assert torch.equal(o8, pkg.fused_moe_fp8(x, w1q, w1s, w2q, w2s, w, ids))
    pkg.check_device_status(cuda_device)


def test_opcheck(cuda_device):
    x, g, bias, w1, w2 = _case(cuda_device, M=16)
    w, ids = pkg.grouped_topk(x, g, 4, True, 4, 2, "sigmoid", 2.5, e_score_correction_bias=bias)
    tests = ("test_schema", "test_faketensor")
    torch.library.opcheck(torch.ops.moe_b200.grouped_topk.default, (x, g, 4, True, 4, 2, "sigmoid", 2.5, bias),
                          test_utils=tests)
    torch.library.opcheck(torch.ops.moe_b200.fused_moe.default, (x, w1, w2, w, ids), test_utils=tests)
    torch.library.opcheck(torch.ops.moe_b200.quantize_rows_fp8.default, (x,), test_utils=tests)


def test_compiled_graph(cuda_device):
    x, g, bias, w1, w2 = _case(cuda_device)

    def layer(xx, gg):
        w, ids = torch.ops.moe_b200.grouped_topk(xx, gg, 4, True, 4, 2, "sigmoid", 2.5, bias)
        return torch.ops.moe_b200.fused_moe(xx, w1, w2, w, ids)

    compiled = torch.compile(layer, fullgraph=True, backend="aot_eager")
    assert torch.equal(compiled(x, g), layer(x, g))


def test_fp8_model_new(cuda_device):
    from test_tasks_cpu import TASKS, load_like_harness

    m = load_like_harness(TASKS / "fused_moe_fp8.py")
    model = m.ModelNew(*m.get_init_inputs()).to(cuda_device)
    torch.manual_seed(42)
    hs, lg = (t.to(cuda_device) for t in m.get_inputs())
    with torch.no_grad():
        a = model(hs, lg)
        b = model(hs, lg)
        assert model.quantizations == 1 and torch.equal(a, b)
        w1q, w1s = pkg.quantize_weights_fp8(model.w1.detach().to(torch.bfloat16))
        w2q, w2s = pkg.quantize_weights_fp8(model.w2.detach().to(torch.bfloat16))
        w, ids = pkg.softmax_topk(lg, 2)
        ref = pkg.fused_moe_fp8(hs.to(torch.bfloat16), w1q, w1s, w2q, w2s, w, ids).to(hs.dtype)
        assert torch.equal(a, ref)
        model.w2.mul_(0.5)  # in-place update: new _version, the FP8 copies are remade
        c = model(hs, lg)
        assert model.quantizations == 2
        torch.testing.assert_close(c.float(), 0.5 * a.float(), atol=2e-3, rtol=5e-2)
    assert a.dtype == hs.dtype and a.shape == hs.shape
