"""numpy restatement of the FP8 w8a8 block-quantised expert path (test infrastructure only).

The reference has no FP8 code (its v0 path is fp16/bf16/fp32 generic,
``fused_moe/v0/fused_moe.py:132,151-152``). The FP8 configuration is defined
as v0 applied to dequantised operands:

* weights: e4m3 with one fp32 scale per 128 x 128 block,
  ``s = amax(|W_block|) / 448`` (1.0 for an all-zero block), ``q = e4m3(W / s)``;
* activations (the token rows, and the SiLU*mul output fed to the down GEMM):
  e4m3 with one fp32 scale per token per 128 channels, same rule;
* the expert path of ``fused_moe/v0/fused_moe.py:141-167`` computed in fp32 on
  ``q * s``.

With ``pow2=True`` (the UE8M0 scale format: DeepSeek's block scales on Blackwell,
the format tcgen05's block-scaled MMA takes) every scale ``amax / 448`` (computed in
fp32) is rounded up to the next power of two, weights and activations alike.

e4m3 here is the OCP FP8 E4M3 format (bias 7, 3 mantissa bits, no infinities,
largest finite 448, subnormals down to 2**-9), rounded to nearest even with
saturation to +-448. This path is parity-unpinned by the reference.
"""

from __future__ import annotations

import numpy as np

E4M3_MAX = np.float32(448.0)


def e4m3_round(v: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest e4m3 value (ties to even), saturating at +-448."""
    v = np.asarray(v, np.float32)
    a = np.minimum(np.abs(v), E4M3_MAX)
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(a > 0, a, np.float32(1.0))))
    e = np.maximum(e, -6.0)                       # below 2**-6: subnormal spacing 2**-9
    quantum = np.exp2(e - 3.0).astype(np.float32)
    q = (np.rint(a / quantum) * quantum).astype(np.float32)
    q = np.minimum(q, E4M3_MAX)
    return np.where(v < 0, -q, q).astype(np.float32)


def _scale(amax: np.ndarray, pow2: bool = False) -> np.ndarray:
    amax = np.asarray(amax, np.float32)
    s = np.where(amax > 0, amax / E4M3_MAX, np.float32(1.0)).astype(np.float32)
    if pow2:  # up to the next power of two: clear the mantissa, one more in the exponent
        b = s.view(np.uint32)
        b = np.where(b & 0x7FFFFF, (b & 0xFF800000) + 0x00800000, b).astype(np.uint32)
        s = b.view(np.float32)
    return s


def quantize_rows_128(x: np.ndarray, pow2: bool = False):
    """Per row, per 128 columns: returns (q fp32-valued e4m3 [M, K], s fp32 [M, K/128])."""
    x = np.asarray(x, np.float32)
    M, K = x.shape
    assert K % 128 == 0
    xb = x.reshape(M, K // 128, 128)
    s = _scale(np.abs(xb).max(axis=-1), pow2)
    q = e4m3_round(xb / s[..., None])
    return q.reshape(M, K), s


def quantize_blocks_128(w: np.ndarray, pow2: bool = False):
    """Per 128 x 128 block of the last two dims: returns (q [..., R, C], s [..., R/128, C/128])."""
    w = np.asarray(w, np.float32)
    *lead, R, C = w.shape
    assert R % 128 == 0 and C % 128 == 0
    wb = w.reshape(*lead, R // 128, 128, C // 128, 128)
    s = _scale(np.abs(wb).max(axis=(-3, -1)), pow2)
    q = e4m3_round(wb / s[..., :, None, :, None])
    return q.reshape(*lead, R, C), s


def dequant_rows(q, s):
    M, K = q.shape
    return (np.asarray(q, np.float32).reshape(M, K // 128, 128) * np.asarray(s)[..., None]).reshape(M, K)


def dequant_blocks(q, s):
    q = np.asarray(q, np.float32)
    *lead, R, C = q.shape
    qb = q.reshape(*lead, R // 128, 128, C // 128, 128)
    return (qb * np.asarray(s)[..., :, None, :, None]).reshape(*lead, R, C)


def moe_experts_fp8_ref(x, w1q, w1s, w2q, w2s, topk_weights, topk_ids, pow2: bool = False):
    """fp32 expert path on dequantised operands; x is quantised per token per 128 here,
    and the SiLU*mul output is quantised the same way before the down projection
    (power-of-two scales for both with pow2)."""
    xq, xs = quantize_rows_128(x, pow2)
    return moe_experts_fp8_rows_ref(xq, xs, w1q, w1s, w2q, w2s, topk_weights, topk_ids, pow2)


def moe_experts_fp8_rows_ref(xq, xs, w1q, w1s, w2q, w2s, topk_weights, topk_ids, pow2: bool = False):
    """``moe_experts_fp8_ref`` from token rows already quantised (xq e4m3 values [M, K],
    xs fp32 [M, K/128]): the expert-parallel FP8 payload. Slots with an id outside
    [0, E) contribute nothing."""
    from .fused_moe import silu

    xd = dequant_rows(xq, xs)
    w1 = dequant_blocks(w1q, w1s)
    w2 = dequant_blocks(w2q, w2s)
    M, K = xd.shape
    N = w1.shape[1] // 2
    ids = np.asarray(topk_ids).astype(np.int64)
    w = np.asarray(topk_weights, np.float32)
    k = ids.shape[1]
    flat = ids.reshape(-1)
    tok = np.repeat(np.arange(M), k)
    y = np.zeros((M * k, K), np.float32)
    for e in np.unique(flat):
        if e < 0 or e >= w1.shape[0]:
            continue
        rows = np.nonzero(flat == e)[0]
        gu = xd[tok[rows]] @ w1[e].T
        act = silu(gu[:, :N]) * gu[:, N:]
        aq, as_ = quantize_rows_128(act, pow2)
        y[rows] = dequant_rows(aq, as_) @ w2[e].T
    valid = (flat >= 0) & (flat < w1.shape[0])
    y *= (w.reshape(-1) * valid)[:, None]
    return y.reshape(M, k, K).sum(axis=1, dtype=np.float32)
