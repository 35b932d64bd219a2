"""fp32 PyTorch restatement of the reference's v0 expert path, for full-size GPU parity checks.

Same steps as ``fused_moe/v0/fused_moe.py:141-167`` (and as ``oracle.fused_moe``),
computed in fp32 on the GPU for a sample of token rows, so DeepSeek-V3-sized
weights (22.5 GB) need not be copied to the host. TF32 is disabled.
"""
import torch


def experts_rows_fp32(x, w1, w2, topk_weights, topk_ids, rows):
    """out[rows] in fp32; x [M,K], w1 [E,2N,K], w2 [E,K,N] (any float dtype, on GPU)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        rows = torch.as_tensor(rows, device=x.device, dtype=torch.long)
        xs = x[rows].float()
        ids = topk_ids[rows].long()
        ws = topk_weights[rows].float()
        N = w1.shape[1] // 2
        out = torch.zeros(len(rows), x.shape[1], dtype=torch.float32, device=x.device)
        for e in torch.unique(ids).tolist():
            r, j = torch.nonzero(ids == e, as_tuple=True)
            gu = xs[r] @ w1[e].float().T
            act = torch.nn.functional.silu(gu[:, :N]) * gu[:, N:]
            y = act @ w2[e].float().T
            out.index_add_(0, r, y * ws[r, j][:, None])
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def _e4m3_rows_128(a, pow2=False):
    """Per row per 128 e4m3 quantise-dequantise (scale = amax / 448, 1 for zero blocks; with
    pow2 rounded up to the next power of two)."""
    M, K = a.shape
    b = a.float().reshape(M, K // 128, 128)
    amax = b.abs().amax(-1, keepdim=True)
    s = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    if pow2:
        bits = s.view(torch.int32)
        up = ((bits & 0x7FFFFF) != 0).to(torch.int32)
        s = ((bits & ~0x7FFFFF) + up * 0x00800000).view(torch.float32)
    return ((b / s).clamp(-448, 448).to(torch.float8_e4m3fn).float() * s).reshape(M, K)


def experts_rows_fp8(x, w1q, w1s, w2q, w2s, topk_weights, topk_ids, rows, pow2=None):
    """fp32 restatement of the FP8 expert path (oracle/fp8.py, exact dequantised operands) for
    sampled token rows, on the GPU. pow2: power-of-two activation scales (the UE8M0 recipe);
    None takes it from the weight scales (all powers of two)."""
    if pow2 is None:
        pow2 = all(bool((((s.float().contiguous().view(torch.int32) & 0x7FFFFF) == 0).all()).item()) for s in (w1s, w2s))
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        rows = torch.as_tensor(rows, device=x.device, dtype=torch.long)
        xs = _e4m3_rows_128(x[rows], pow2)
        ids = topk_ids[rows].long()
        ws = topk_weights[rows].float()
        E, twoN, K = w1q.shape
        N = twoN // 2
        out = torch.zeros(len(rows), K, dtype=torch.float32, device=x.device)
        for e in torch.unique(ids).tolist():
            r, j = torch.nonzero(ids == e, as_tuple=True)
            w1 = (w1q[e].float().reshape(twoN // 128, 128, K // 128, 128) * w1s[e][:, None, :, None]).reshape(twoN, K)
            w2 = (w2q[e].float().reshape(K // 128, 128, N // 128, 128) * w2s[e][:, None, :, None]).reshape(K, N)
            gu = xs[r] @ w1.T
            act = _e4m3_rows_128(torch.nn.functional.silu(gu[:, :N]) * gu[:, N:], pow2)
            out.index_add_(0, r, (act @ w2.T) * ws[r, j][:, None])
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
