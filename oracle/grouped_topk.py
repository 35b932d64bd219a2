"""numpy restatement of the reference's routing rules (test infrastructure only).

``grouped_topk_ref`` follows ``grouped_topk/v0/grouped_topk.py:91-132`` of the
reference step by step:

1. scores = softmax(g) or sigmoid(g)                          (v0 :98-103)
2. group score = max of the group's scores                    (v0 :109-111)
3. keep the ``topk_group`` best groups                        (v0 :112)
4. mask the experts of the other groups with -inf             (v0 :115-123)
5. top-k experts, sorted descending                           (v0 :124)
6. renormalise                                                (v0 :126-127)
7. multiply by ``routed_scaling_factor`` when it is not 1.0   (v0 :129-130)

Extension (DeepSeek-V3 routing, not implemented by the reference): with
``e_score_correction_bias`` the ranking in steps 2-5 uses ``scores + bias``
while the returned weights are gathered from ``scores`` without the bias; with
``group_score="top2sum"`` step 2 uses the sum of the two best values in each
group. With bias=None and group_score="max" the function is exactly v0.

Ties. ``torch.topk`` leaves the order of equal values undefined (the reference
says so at ``grouped_topk/v0/grouped_topk.py:20-29``). This oracle, like the CUDA
kernel, uses the strict total order (value descending, index ascending), which
is the rank rule of the reference's Triton kernel
(``grouped_topk/v1/grouped_topk.py:94``). Rows whose selection boundary holds a
tie can therefore differ from v0; ``boundary_margin`` reports them.

``softmax_topk_ref`` follows the routing block of
``fused_moe/v0/fused_moe.py:134-139`` (softmax in fp32, top-k, renormalise,
cast of the weights to the hidden dtype left to the caller).
"""

from __future__ import annotations

import numpy as np


def _scores(g: np.ndarray, scoring_func: str) -> np.ndarray:
    g = np.asarray(g, dtype=np.float32)
    if scoring_func == "softmax":
        m = g.max(axis=-1, keepdims=True)
        e = np.exp(g - m, dtype=np.float32)
        return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    if scoring_func == "sigmoid":
        return (np.float32(1.0) / (np.float32(1.0) + np.exp(-g, dtype=np.float32))).astype(np.float32)
    raise ValueError(f"Unsupported scoring_func: {scoring_func}")


def _rank_desc(v: np.ndarray) -> np.ndarray:
    """Indices that sort each row by (value descending, index ascending)."""
    return np.argsort(-v, axis=-1, kind="stable")


def grouped_topk_ref(
    gating_output: np.ndarray,
    topk: int,
    renormalize: bool,
    num_expert_group: int,
    topk_group: int,
    scoring_func: str = "softmax",
    routed_scaling_factor: float = 1.0,
    e_score_correction_bias: np.ndarray | None = None,
    group_score: str = "max",
):
    """Returns (topk_weights float32 [M, topk], topk_ids int32 [M, topk])."""
    g = np.asarray(gating_output, dtype=np.float32)
    M, E = g.shape
    if E % num_expert_group:
        raise ValueError("num_experts must be divisible by num_expert_group")
    epg = E // num_expert_group
    scores = _scores(g, scoring_func)                                  # v0 :98-103
    if e_score_correction_bias is not None:
        choice = (scores + np.asarray(e_score_correction_bias, np.float32)[None, :]).astype(np.float32)
    else:
        choice = scores
    grouped = choice.reshape(M, num_expert_group, epg)
    if group_score == "max":
        gscore = grouped.max(axis=-1)                                   # v0 :109-111
    elif group_score == "top2sum":
        top2 = -np.sort(-grouped, axis=-1)[..., :2]
        gscore = (top2[..., 0] + top2[..., 1]).astype(np.float32)
    else:
        raise ValueError(f"Unsupported group_score: {group_score}")
    group_idx = _rank_desc(gscore)[:, :topk_group]                     # v0 :112
    group_mask = np.zeros((M, num_expert_group), dtype=bool)
    np.put_along_axis(group_mask, group_idx, True, axis=1)             # v0 :115-116
    score_mask = np.repeat(group_mask, epg, axis=1)                    # v0 :117-121
    masked = np.where(score_mask, choice, np.float32(-np.inf))          # v0 :123
    ids = _rank_desc(masked)[:, :topk]                                 # v0 :124
    w = np.take_along_axis(scores, ids, axis=1).astype(np.float32)
    if renormalize:                                                    # v0 :126-127
        w = (w / w.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    if routed_scaling_factor != 1.0:                                   # v0 :129-130
        w = (w * np.float32(routed_scaling_factor)).astype(np.float32)
    return w.astype(np.float32), ids.astype(np.int32)


def boundary_margin(
    gating_output: np.ndarray,
    topk: int,
    num_expert_group: int,
    topk_group: int,
    scoring_func: str = "softmax",
    e_score_correction_bias: np.ndarray | None = None,
    group_score: str = "max",
) -> np.ndarray:
    """Per row, the smallest gap at a selection boundary (group and expert).

    A row whose gap is within a few ulp may legitimately select differently on
    hardware whose exp differs by 1 ulp, or under torch.topk's undefined tie
    order; parity tests report such rows separately.
    """
    g = np.asarray(gating_output, dtype=np.float32)
    M, E = g.shape
    epg = E // num_expert_group
    scores = _scores(g, scoring_func)
    choice = scores if e_score_correction_bias is None else (
        scores + np.asarray(e_score_correction_bias, np.float32)[None, :])
    grouped = choice.reshape(M, num_expert_group, epg)
    if group_score == "max":
        gscore = grouped.max(axis=-1)
    else:
        top2 = -np.sort(-grouped, axis=-1)[..., :2]
        gscore = top2[..., 0] + top2[..., 1]
    gs = -np.sort(-gscore, axis=-1)
    gap_g = (gs[:, topk_group - 1] - gs[:, topk_group]) if topk_group < num_expert_group else np.full(M, np.inf)
    group_idx = _rank_desc(gscore)[:, :topk_group]
    mask = np.zeros((M, num_expert_group), dtype=bool)
    np.put_along_axis(mask, group_idx, True, axis=1)
    masked = np.where(np.repeat(mask, epg, axis=1), choice, -np.inf)
    ms = -np.sort(-masked, axis=-1)
    gap_e = ms[:, topk - 1] - ms[:, topk] if topk < E else np.full(M, np.inf)
    gap_e = np.where(np.isfinite(gap_e), gap_e, np.inf)
    # within-top-k ordering ties also change the order of ids
    inner = np.min(np.abs(np.diff(ms[:, :topk], axis=-1)), axis=-1) if topk > 1 else np.full(M, np.inf)
    return np.minimum(np.minimum(np.abs(gap_g), np.abs(gap_e)), inner)


def softmax_topk_ref(router_logits: np.ndarray, top_k: int, renormalize: bool = True):
    """Mixtral routing of ``fused_moe/v0/fused_moe.py:134-139`` (weights in fp32)."""
    scores = _scores(np.asarray(router_logits, np.float32), "softmax")  # :135
    ids = _rank_desc(scores)[:, :top_k]                                  # :136
    w = np.take_along_axis(scores, ids, axis=1)
    if renormalize:                                                      # :137-138
        w = (w / w.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return w.astype(np.float32), ids.astype(np.int32)
