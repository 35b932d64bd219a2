"""CPU: the threshold top-k selection of the E = 256 routing kernel, restated in numpy,
against the oracle.

The kernel (csrc/routing.cuh, route_select_threshold8) takes the top-k of the kept groups
only from the values at or above t, the smallest second-best value among the kept groups,
because the kept groups' two best values are 2 * topk_group >= k values all >= t. This
test restates that selection step by step (group ranking by score descending and group
index ascending, threshold, candidates compacted in lane order, rank by the number of
larger (value, -index) keys) and checks it against grouped_topk_ref on Gaussian,
skewed-bias and tie-heavy logits, rows with more than 32 candidates included (where the
kernel takes its fallback selection, which here is the oracle itself).
"""
import numpy as np
import pytest

from oracle.grouped_topk import _scores, grouped_topk_ref


def _threshold_topk(g, topk, n_group, topk_group, bias, group_score, scale):
    """Returns (weights, ids, n_candidates) per the kernel's threshold path; ids None where
    more than 32 values pass (the kernel's fallback)."""
    M, E = g.shape
    epg = E // n_group
    s = _scores(g, "sigmoid")
    c = (s + bias[None, :]).astype(np.float32) if bias is not None else s
    grouped = c.reshape(M, n_group, epg)
    top2 = -np.sort(-grouped, axis=-1)[..., :2]
    b1, b2 = top2[..., 0], top2[..., 1]
    gs = b1 if group_score == "max" else (b1 + b2).astype(np.float32)
    out_w = np.zeros((M, topk), np.float32)
    out_i = np.full((M, topk), -1, np.int32)
    ncand = np.zeros(M, np.int64)
    for m in range(M):
        # kept groups: topk_group rounds of (largest remaining score, lowest group holding it)
        kept = []
        for _ in range(topk_group):
            rest = [h for h in range(n_group) if h not in kept]
            best = max(gs[m, h] for h in rest)
            kept.append(min(h for h in rest if gs[m, h] == best))
        t = min(b2[m, h] for h in kept)
        cand = [e for h in sorted(kept) for e in range(h * epg, (h + 1) * epg) if not (c[m, e] < t)]
        ncand[m] = len(cand)
        assert len(cand) >= 2 * topk_group >= topk
        if len(cand) > 32:
            out_i[m] = -2  # fallback row
            continue
        rank = {e: sum(1 for f in cand if (c[m, f], -f) > (c[m, e], -e)) for e in cand}
        chosen = sorted((r, e) for e, r in rank.items() if r < topk)
        ids = [e for _, e in chosen]
        w = np.array([s[m, e] for e in ids], np.float32)
        w = (w / w.sum(dtype=np.float32)).astype(np.float32) * np.float32(scale)
        out_i[m] = ids
        out_w[m] = w
    return out_w, out_i, ncand


@pytest.mark.parametrize("kind", ["gaussian", "skewed", "ties"])
@pytest.mark.parametrize("group_score", ["top2sum", "max"])
def test_threshold_selection_equals_full_topk(kind, group_score):
    rng = np.random.default_rng({"gaussian": 1, "skewed": 2, "ties": 3}[kind])
    M = 300
    if kind == "ties":
        g = (rng.integers(-2, 3, size=(M, 256)) / 2).astype(np.float32)
        g[::7] = 0.25  # every expert ties: more than 32 candidates
        bias = (rng.integers(0, 2, size=256) * 0.01).astype(np.float32)
    else:
        g = rng.standard_normal((M, 256)).astype(np.float32)
        bias = (rng.standard_normal(256) * 0.01).astype(np.float32)
        if kind == "skewed":
            bias[rng.permutation(256)[:16]] = 2.0
    w, ids, ncand = _threshold_topk(g, 8, 8, 4, bias, group_score, 2.5)
    rw, rids = grouped_topk_ref(g, 8, True, 8, 4, "sigmoid", 2.5, e_score_correction_bias=bias,
                                group_score=group_score)
    fast = ids[:, 0] != -2
    np.testing.assert_array_equal(ids[fast], rids[fast])
    np.testing.assert_allclose(w[fast], rw[fast], rtol=0, atol=1e-6)
    if kind == "gaussian":
        assert fast.all() and ncand.max() <= 32  # the fast path covers Gaussian logits
    if kind == "ties":
        assert (~fast).any()  # constant rows take the fallback
