"""HostPipeline: batches in pinned host memory give the same bits as the layer called batch by batch."""
import pytest
import torch

from kernelswift_competition_submission_b200 import check_device_status, moe_layer
from kernelswift_competition_submission_b200.pipeline import HostPipeline

pytestmark = pytest.mark.gpu


def test_pipeline_matches_sequential(cuda_device):
    dev = cuda_device
    E, K, N, M, k = 16, 256, 128, 96, 4
    gen = torch.Generator(device=dev).manual_seed(5)
    w1 = (torch.randn(E, 2 * N, K, generator=gen, device=dev) / K ** 0.5).to(torch.bfloat16)
    w2 = (torch.randn(E, K, N, generator=gen, device=dev) / N ** 0.5).to(torch.bfloat16)
    bias = torch.randn(E, generator=gen, device=dev) * 0.01

    def fn(x, g):
        return moe_layer(x, g, w1, w2, topk=k, renormalize=True, num_expert_group=4, topk_group=2,
                         scoring_func="sigmoid", routed_scaling_factor=2.5, e_score_correction_bias=bias)

    n = 5
    xs = [torch.randn(M, K, generator=gen, device=dev).to(torch.bfloat16).cpu().pin_memory() for _ in range(n)]
    gs = [torch.randn(M, E, generator=gen, device=dev).cpu().pin_memory() for _ in range(n)]
    outs = [torch.empty(M, K, dtype=torch.bfloat16).pin_memory() for _ in range(n)]
    HostPipeline(fn, dev).run(xs, gs, outs)
    for i in range(n):
        want = fn(xs[i].to(dev), gs[i].to(dev)).cpu()
        assert torch.equal(outs[i], want), i
    check_device_status(dev)


def test_pipeline_rejects_pageable(cuda_device):
    p = HostPipeline(lambda x, g: x, cuda_device)
    with pytest.raises(ValueError):
        p.run([torch.zeros(4, 4)], [torch.zeros(4, 4)], [torch.zeros(4, 4)])
