"""GPU: router GEMM fused with grouped_topk (moe_router_grouped_topk).

Logits against an fp32 matmul of the same bf16/fp16 operands (atol = rtol = 1e-4: the
products are exact in fp32, only the summation order differs); the routing against
grouped_topk run on the fused kernel's own logits, bit-exact (same rule, same values)."""
import pytest
import torch

from kernelswift_competition_submission_b200 import check_device_status, grouped_topk, router_grouped_topk

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,K,dtype,scoring,bias,groups", [
    (1, 7168, torch.bfloat16, "sigmoid", True, (8, 4)),      # decode: one m-block split over many CTAs
    (83, 512, torch.float16, "softmax", False, (8, 4)),
    (128, 7168, torch.bfloat16, "sigmoid", True, (8, 4)),
    (300, 1024, torch.bfloat16, "softmax", False, (1, 1)),   # ragged m-blocks, no group mask
    (4096, 7168, torch.bfloat16, "sigmoid", True, (8, 4)),   # prefill: one CTA per m-block
    (257, 2048, torch.bfloat16, "sigmoid", True, (16, 8)),   # 16 experts per group (2 lanes)
])
def test_router_fused_matches(cuda_device, M, K, dtype, scoring, bias, groups):
    dev = cuda_device
    gen = torch.Generator(device=dev).manual_seed(M + K)
    x = torch.randn(M, K, generator=gen, device=dev).to(dtype)
    wg = (torch.randn(256, K, generator=gen, device=dev) / K ** 0.5).to(dtype)
    b = torch.randn(256, generator=gen, device=dev) * 0.01 if bias else None
    ng, tg = groups
    w, ids, logits = router_grouped_topk(x, wg, 8, True, ng, tg, scoring, 2.5, e_score_correction_bias=b,
                                         return_logits=True)
    ref_logits = x.float() @ wg.float().T
    torch.testing.assert_close(logits, ref_logits, atol=1e-4, rtol=1e-4)
    w2, ids2 = grouped_topk(x, logits, 8, True, ng, tg, scoring, 2.5, e_score_correction_bias=b)
    assert torch.equal(ids, ids2)
    assert torch.equal(w, w2)
    check_device_status(dev)


def test_router_rejects_other_expert_counts(cuda_device):
    x = torch.randn(4, 128, device=cuda_device).bfloat16()
    wg = torch.randn(128, 128, device=cuda_device).bfloat16()
    with pytest.raises(RuntimeError):
        router_grouped_topk(x, wg, 8, True, 8, 4, "sigmoid", 1.0)
