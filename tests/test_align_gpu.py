"""GPU parity of the align stage (counting sort by expert) against the oracle."""
import numpy as np
import pytest
import torch

from kernelswift_competition_submission_b200 import moe_align
from oracle.fused_moe import moe_align_ref

pytestmark = pytest.mark.gpu


def _check(ids_np, E, bm, dev):
    counts, bs, sp = moe_align(torch.from_numpy(ids_np).to(dev), E, bm)
    torch.cuda.synchronize()
    r = moe_align_ref(ids_np, E, bm)
    np.testing.assert_array_equal(counts.cpu().numpy(), r["counts"])
    np.testing.assert_array_equal(bs.cpu().numpy(), r["block_start"])
    sp = sp.cpu().numpy()
    total = int(r["block_start"][-1]) * bm
    for e in range(E):
        a, b = int(r["block_start"][e]) * bm, int(r["block_start"][e + 1]) * bm
        np.testing.assert_array_equal(np.sort(sp[a:a + r["counts"][e]]), np.sort(r["sorted_pairs"][a:a + r["counts"][e]]))
        assert (sp[a + r["counts"][e]:b] == -1).all()
    assert np.array_equal(np.sort(sp[:total][sp[:total] >= 0]), np.arange(ids_np.size))


@pytest.mark.parametrize("M,E,k", [(1, 256, 8), (83, 8, 2), (4096, 256, 8), (32768, 256, 8), (777, 1024, 3)])
def test_uniform(cuda_device, M, E, k):
    rng = np.random.default_rng(M)
    _check(rng.integers(0, E, size=(M, k)).astype(np.int32), E, 128, cuda_device)


def test_all_pairs_one_expert(cuda_device):
    _check(np.full((1000, 2), 5, np.int32), 8, 128, cuda_device)


def test_skewed_and_empty_experts(cuda_device):
    rng = np.random.default_rng(9)
    ids = rng.integers(0, 16, size=(5000, 8)).astype(np.int32)  # experts 16..255 empty
    _check(ids, 256, 128, cuda_device)


def test_empty(cuda_device):
    counts, bs, sp = moe_align(torch.empty(0, 8, dtype=torch.int32, device=cuda_device), 8, 128)
    assert int(counts.sum()) == 0 and int(bs[-1]) == 0
