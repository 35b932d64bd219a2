"""GPU: the expert-parallel dispatch/combine kernels against the torch restatement of the plan.

One GPU is enough: the kernels only plan, pack and combine; the exchange between
ranks is NCCL's. ``plan_dispatch`` (the plan the CPU/gloo tests use) is the reference.
"""
import pytest
import torch

from kernelswift_competition_submission_b200 import _lib
from kernelswift_competition_submission_b200.ep import plan_dispatch
from kernelswift_competition_submission_b200.ops import _DTYPES, _ptr, _stream

pytestmark = pytest.mark.gpu


def _run(M, K, topk, E, world, dtype, dev, seed=0):
    gen = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, K, generator=gen, device=dev).to(dtype)
    ids = torch.stack([torch.randperm(E, generator=gen, device=dev)[:topk] for _ in range(M)]).to(torch.int32) \
        if M else torch.empty(0, topk, dtype=torch.int32, device=dev)
    if M:
        ids[::7, 0] = -1  # some slots routed nowhere
    w = torch.rand(M, topk, generator=gen, device=dev)
    epr = E // world
    lib = _lib.load()
    cap = max(1, lib.moe_ep_send_capacity(M, topk, world))
    send_x = torch.empty(cap, K, dtype=dtype, device=dev)
    meta = torch.empty(cap, 2 * topk, dtype=torch.int32, device=dev)
    scratch = torch.empty(2 * world + 1, dtype=torch.int32, device=dev)
    offsets = torch.empty(world + 1, dtype=torch.int32, device=dev)
    counts = torch.empty(world, dtype=torch.int64, device=dev)
    tok_rows = torch.empty(max(M, 1), world, dtype=torch.int32, device=dev)
    st = _stream(dev)
    _lib.check(lib.moe_ep_plan(_ptr(ids), M, topk, epr, world, _ptr(scratch), _ptr(offsets), _ptr(counts), st), "plan")
    _lib.check(lib.moe_ep_pack(_DTYPES[dtype], _ptr(x), _ptr(ids), _ptr(w), M, K, topk, epr, world, _ptr(scratch),
                               _ptr(offsets), _ptr(send_x), _ptr(meta), _ptr(tok_rows), st), "pack")
    torch.cuda.synchronize()
    ref_tok, ref_counts, ref_ids, ref_w = plan_dispatch(ids, w, epr, world)
    assert counts.tolist() == ref_counts.tolist()
    S = int(ref_counts.sum())
    assert int(offsets[-1]) == S
    # every (token, destination) row: right token data, right metadata, inside its destination block
    ref_rows = {}
    for i, (t, d) in enumerate(zip(ref_tok.tolist(), torch.repeat_interleave(torch.arange(world), ref_counts.cpu()).tolist())):
        ref_rows[(t, d)] = i
    tr = tok_rows[:M].cpu()
    off = offsets.cpu()
    for t in range(M):
        for d in range(world):
            row = int(tr[t, d])
            if (t, d) not in ref_rows:
                assert row == -1
                continue
            assert int(off[d]) <= row < int(off[d + 1])
            i = ref_rows[(t, d)]
            assert torch.equal(send_x[row], x[t])
            assert torch.equal(meta[row, :topk], ref_ids[i])
            assert torch.equal(meta[row, topk:].view(torch.float32), ref_w[i])
    # combine: out[t] = sum over its destinations of the returned rows
    back = torch.randn(max(S, 1), K, generator=gen, device=dev).to(dtype)
    out = torch.empty(M, K, dtype=dtype, device=dev)
    _lib.check(lib.moe_ep_combine(_DTYPES[dtype], _ptr(back), _ptr(tok_rows), M, K, world, _ptr(out), st), "combine")
    ref = torch.zeros(M, K, dtype=torch.float32, device=dev)
    for (t, d), i in ref_rows.items():
        ref[t] += back[int(tr[t, d])].float()
    torch.testing.assert_close(out.float(), ref.to(dtype).float(), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("M,K,topk,E,world,dtype", [(97, 256, 8, 64, 8, torch.bfloat16),
                                                     (40, 128, 2, 8, 4, torch.float16),
                                                     (33, 512, 6, 32, 2, torch.bfloat16),
                                                     (5, 64, 4, 64, 64, torch.bfloat16)])
def test_ep_kernels_match_plan(cuda_device, M, K, topk, E, world, dtype):
    _run(M, K, topk, E, world, dtype, cuda_device)


def test_ep_kernels_empty(cuda_device):
    _run(0, 128, 8, 64, 8, torch.bfloat16, cuda_device)
