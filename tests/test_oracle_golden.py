"""CPU: the numpy oracle against golden vectors produced by the reference's own v0 code."""
import numpy as np
import pytest

from oracle.fused_moe import fused_moe_layer_ref, moe_align_ref, moe_experts_ref, to_bf16
from oracle.grouped_topk import boundary_margin, grouped_topk_ref, softmax_topk_ref

GT_FILES = [
    "grouped_topk_task.npz",
    "grouped_topk_sigmoid_m128.npz",
    "grouped_topk_ragged_m1.npz",
    "grouped_topk_m37_e128.npz",
    "grouped_topk_mixtral_m256.npz",
    "grouped_topk_m300_e256_k8.npz",
]


def _gt_args(d):
    return dict(topk=int(d["topk"]), renormalize=bool(d["renormalize"]),
                num_expert_group=int(d["num_expert_group"]), topk_group=int(d["topk_group"]),
                scoring_func=str(d["scoring_func"]), routed_scaling_factor=float(d["routed_scaling_factor"]))


@pytest.mark.parametrize("name", GT_FILES)
def test_grouped_topk_oracle_matches_v0(golden_dir, name):
    d = np.load(golden_dir / name)
    w, ids = grouped_topk_ref(d["gating_output"], **_gt_args(d))
    np.testing.assert_array_equal(ids, d["topk_ids"])
    np.testing.assert_allclose(w, d["topk_weights"], rtol=0, atol=1e-6)


def test_bias_extension_reduces_to_v0(golden_dir):
    d = np.load(golden_dir / "grouped_topk_sigmoid_m128.npz")
    a = _gt_args(d)
    w0, i0 = grouped_topk_ref(d["gating_output"], **a)
    w1, i1 = grouped_topk_ref(d["gating_output"], **a, e_score_correction_bias=np.zeros(256, np.float32),
                              group_score="max")
    np.testing.assert_array_equal(i0, i1)
    np.testing.assert_array_equal(w0, w1)


def test_bias_changes_selection_not_weights_source():
    rng = np.random.default_rng(0)
    g = rng.standard_normal((64, 256), dtype=np.float32)
    bias = np.zeros(256, np.float32)
    bias[:16] = 2.0  # hot experts
    w, ids = grouped_topk_ref(g, 8, False, 8, 4, "sigmoid", 1.0, bias, "top2sum")
    assert (ids < 16).mean() > 0.5
    sig = 1.0 / (1.0 + np.exp(-g))
    np.testing.assert_allclose(w, np.take_along_axis(sig, ids, 1), rtol=1e-6)


def test_mixtral_routing_is_grouped_topk_special_case(golden_dir):
    d = np.load(golden_dir / "grouped_topk_mixtral_m256.npz")
    w, ids = softmax_topk_ref(d["gating_output"], 2, True)
    np.testing.assert_array_equal(ids, d["topk_ids"])
    np.testing.assert_allclose(w, d["topk_weights"], atol=1e-6)


def test_boundary_margin_flags_ties():
    g = np.zeros((2, 16), np.float32)
    g[1] = np.arange(16, dtype=np.float32)
    m = boundary_margin(g, 4, 4, 2, "softmax")
    assert m[0] == 0.0 and m[1] > 0.0


@pytest.mark.parametrize("name,key,tol", [("fused_moe_task.npz", "out_fp32", 1e-6),
                                          ("fused_moe_small_fp32.npz", "out_fp32", 1e-6)])
def test_fused_moe_oracle_matches_v0(golden_dir, name, key, tol):
    d = np.load(golden_dir / name)
    out, _, _ = fused_moe_layer_ref(d["hidden_states"].astype(np.float32), d["router_logits"],
                                    d["w1"].astype(np.float32), d["w2"].astype(np.float32), int(d["top_k"]))
    np.testing.assert_allclose(out, d[key], rtol=1e-4, atol=tol)


def test_fused_moe_oracle_close_to_v0_fp16(golden_dir):
    d = np.load(golden_dir / "fused_moe_task.npz")
    out, _, _ = fused_moe_layer_ref(d["hidden_states"].astype(np.float32), d["router_logits"],
                                    d["w1"].astype(np.float32), d["w2"].astype(np.float32), int(d["top_k"]))
    np.testing.assert_allclose(out, d["out_fp16"].astype(np.float32), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("M,E,k,bm", [(0, 8, 2, 128), (1, 256, 8, 128), (83, 8, 2, 128), (513, 64, 6, 128),
                                      (1000, 3, 1, 64)])
def test_align_oracle_against_brute_force(M, E, k, bm):
    rng = np.random.default_rng(M + E)
    ids = rng.integers(0, E, size=(M, k)).astype(np.int32)
    r = moe_align_ref(ids, E, bm)
    flat = ids.reshape(-1)
    for e in range(E):
        rows = r["sorted_pairs"][r["block_start"][e] * bm:r["block_start"][e + 1] * bm]
        got = sorted(int(p) for p in rows if p >= 0)
        assert got == sorted(np.nonzero(flat == e)[0].tolist())
        assert (rows[len(got):] == -1).all()
    assert r["counts"].sum() == M * k
    assert (np.diff(r["block_start"]) == (r["counts"] + bm - 1) // bm).all()
    assert len(r["block_expert"]) == r["block_start"][-1]


def test_expert_path_per_row_independence():
    rng = np.random.default_rng(1)
    M, E, k, K, N = 20, 4, 2, 32, 16
    x = rng.standard_normal((M, K), dtype=np.float32)
    w1 = rng.standard_normal((E, 2 * N, K), dtype=np.float32) * 0.1
    w2 = rng.standard_normal((E, K, N), dtype=np.float32) * 0.1
    ids = rng.integers(0, E, size=(M, k)).astype(np.int32)
    w = rng.random((M, k), dtype=np.float32)
    full = moe_experts_ref(x, w1, w2, w, ids)
    rows = [3, 7, 19]
    part = moe_experts_ref(x[rows], w1, w2, w[rows], ids[rows])
    np.testing.assert_allclose(part, full[rows], rtol=1e-6, atol=1e-6)


def test_to_bf16_rounding():
    a = np.array([1.0, 1.00390625, 1.005859375, -3.3e-3, np.inf], np.float32)
    b = to_bf16(a)
    assert b[0] == 1.0 and b[1] == 1.0 and b[2] == np.float32(1.0078125) and np.isinf(b[4])
