"""numpy restatement of the reference's ``fused_moe`` expert path (test infrastructure only).

``moe_experts_ref`` follows ``fused_moe/v0/fused_moe.py:141-167``:

* every (token, slot) pair is an independent row                  (:143-149)
* per expert e: ``gate_up = x_e @ w1[e].T``; ``gate, up = chunk(2)``  (:160-161)
  (gate = columns [0, I), up = columns [I, 2I))
* ``act = silu(gate) * up``; ``y = act @ w2[e].T``                   (:162-163)
* ``out[t] = sum_j w[t, j] * y[t, j]``                                (:166-167)

v0 computes in the hidden dtype; this restatement accumulates in fp32 on the
same (already rounded) operands, which is the "fp32-accumulated reference" the
parity tolerances are stated against. With fp32 inputs it is v0 itself.

``moe_align_ref`` is the oracle of the CUDA align stage, which the reference
does not have (v0 uses a per-expert boolean mask, ``fused_moe/v0/fused_moe.py:155-159``):
a stable counting sort of the pairs by expert, each expert's segment padded up
to a multiple of ``block_m``.
"""

from __future__ import annotations

import numpy as np


def silu(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def to_bf16(a: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bfloat16 (ties to even); returned as fp32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(a), a, out).astype(np.float32)


def moe_experts_ref(x, w1, w2, topk_weights, topk_ids):
    """fp32 expert path of v0 for all tokens. x [M,K], w1 [E,2N,K], w2 [E,K,N]."""
    x = np.asarray(x, np.float32)
    M, K = x.shape
    E, twoN, _ = w1.shape
    N = twoN // 2
    ids = np.asarray(topk_ids).astype(np.int64)
    w = np.asarray(topk_weights, np.float32)
    k = ids.shape[1]
    flat_ids = ids.reshape(-1)                                          # :143
    flat_w = w.reshape(-1)                                              # :144
    tok = np.repeat(np.arange(M), k)                                    # :145-149 (x_rep)
    y = np.zeros((M * k, K), np.float32)
    for e in np.unique(flat_ids):                                       # :155-158
        rows = np.nonzero(flat_ids == e)[0]
        xe = x[tok[rows]]                                               # :159
        gu = xe @ np.asarray(w1[e], np.float32).T                       # :160
        act = silu(gu[:, :N]) * gu[:, N:]                               # :161-162
        y[rows] = act @ np.asarray(w2[e], np.float32).T                 # :163
    y *= flat_w[:, None]                                                # :166
    return y.reshape(M, k, K).sum(axis=1, dtype=np.float32)             # :167


def moe_experts_rows_ref(x, w1, w2, topk_weights, topk_ids, rows):
    """Same as ``moe_experts_ref`` restricted to token indices ``rows``.

    Each output row depends only on its own token, so a seeded sample of rows
    checks a full-size launch at a fraction of the CPU cost.
    """
    rows = np.asarray(rows, np.int64)
    return moe_experts_ref(np.asarray(x, np.float32)[rows], w1, w2,
                           np.asarray(topk_weights)[rows], np.asarray(topk_ids)[rows])


def moe_align_ref(topk_ids, num_experts: int, block_m: int):
    """Counting sort of (token, slot) pairs by expert, padded per expert.

    Returns a dict with
      counts       int32 [E]      pairs routed to each expert
      block_start  int32 [E + 1]  first m-block of each expert (prefix sum of ceil(count/block_m))
      sorted_pairs int32 [R]      pair id (token * topk + slot) per padded row, -1 in padding
      block_expert int32 [B]      expert of each m-block
    """
    flat = np.asarray(topk_ids).astype(np.int64).reshape(-1)
    counts = np.bincount(flat, minlength=num_experts)[:num_experts].astype(np.int64)
    nblk = (counts + block_m - 1) // block_m
    block_start = np.zeros(num_experts + 1, np.int64)
    block_start[1:] = np.cumsum(nblk)
    R = int(block_start[-1]) * block_m
    sorted_pairs = np.full(R, -1, np.int64)
    order = np.argsort(flat, kind="stable")
    pos = 0
    for e in range(num_experts):
        c = int(counts[e])
        base = int(block_start[e]) * block_m
        sorted_pairs[base:base + c] = order[pos:pos + c]
        pos += c
    block_expert = np.repeat(np.arange(num_experts), nblk)
    return {
        "counts": counts.astype(np.int32),
        "block_start": block_start.astype(np.int32),
        "sorted_pairs": sorted_pairs.astype(np.int32),
        "block_expert": block_expert.astype(np.int32),
    }


def fused_moe_layer_ref(x, router_logits, w1, w2, top_k: int, renormalize: bool = True):
    """The whole Mixtral-style layer of ``fused_moe/v0/fused_moe.py:126-167`` in fp32."""
    from .grouped_topk import softmax_topk_ref

    w, ids = softmax_topk_ref(router_logits, top_k, renormalize)
    return moe_experts_ref(x, w1, w2, w, ids), w, ids
