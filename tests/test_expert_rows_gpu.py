"""GPU: every output row of the expert path at awkward per-expert row counts.

Experts with no rows, one row, 129, 257 and 385 rows (1, 2 and 3 full m-blocks of 128
plus one row, so the last m-block of each is nearly empty), the rest random; bf16 and
fp16; hidden sizes with a ragged last down-GEMM n-block. All rows are checked against the
fp32 restatement of the reference's expert path (fused_moe/v0/fused_moe.py:141-167), and a
second call must give the same bits.
"""
import pytest
import torch

from kernelswift_competition_submission_b200 import check_device_status, fused_moe
from torch_ref import experts_rows_fp32

pytestmark = pytest.mark.gpu


def _ids_with_shapes(M, E, k, dev, seed):
    """topk ids where expert 0 has no pair, expert 1 one pair, experts 2-4 have
    129, 257 and 385 pairs (odd and even m-block counts), the rest random."""
    assert E - 5 >= k, "needs k distinct experts among 5 .. E-1"
    gen = torch.Generator(device=dev).manual_seed(seed)
    ids = torch.randint(5, E, (M, k), generator=gen, device=dev, dtype=torch.int32)
    want = {1: 1, 2: 129, 3: 257, 4: 385}
    t = 0
    for e, n in want.items():  # slot 0 of consecutive tokens; the other slots hold experts >= 5
        ids[t:t + n, 0] = e
        t += n
    # a token never repeats an expert: redraw repeated slots among experts >= 5
    rows = ids.cpu()
    for r in range(M):
        seen = set()
        for j in range(k):
            e = int(rows[r, j])
            while e in seen:
                e = 5 + (e - 5 + 1) % (E - 5)
            rows[r, j] = e
            seen.add(e)
    return rows.to(dev)


@pytest.mark.parametrize("M,E,k,K,N,dtype", [(3000, 8, 2, 512, 256, torch.bfloat16),
                                             (2600, 16, 4, 320, 128, torch.bfloat16),
                                             (3000, 8, 2, 256, 384, torch.float16),
                                             (9000, 16, 4, 1024, 512, torch.bfloat16)])
def test_all_rows_awkward_counts(cuda_device, M, E, k, K, N, dtype):
    dev = cuda_device
    gen = torch.Generator(device=dev).manual_seed(M + K)
    x = torch.randn(M, K, generator=gen, device=dev).to(dtype)
    w1 = (torch.randn(E, 2 * N, K, generator=gen, device=dev) / K ** 0.5).to(dtype)
    w2 = (torch.randn(E, K, N, generator=gen, device=dev) / N ** 0.5).to(dtype)
    ids = _ids_with_shapes(M, E, k, dev, seed=M)
    w = torch.rand(M, k, generator=gen, device=dev)
    counts = torch.bincount(ids.flatten().long(), minlength=E)
    assert counts[0] == 0 and counts[1] == 1 and counts[2] == 129 and counts[3] == 257
    out = fused_moe(x, w1, w2, w, ids)
    torch.cuda.synchronize()
    check_device_status(dev)
    ref = experts_rows_fp32(x, w1, w2, w, ids, torch.arange(M))
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
    again = fused_moe(x, w1, w2, w, ids)
    assert torch.equal(out, again)
