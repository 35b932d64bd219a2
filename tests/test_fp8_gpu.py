"""GPU parity of the FP8 w8a8 path: e4m3 quantisers (bit-exact against the oracle) and the
fused FP8 expert path (atol = rtol = 5e-2 elementwise against the oracle's fp32 expert path on
the exact dequantised operands, and 1e-2 on the aggregate relative error), with fp32 block
scales (promotion GEMMs) and with power-of-two UE8M0 scales (block-scaled GEMMs at prefill
sizes, the promotion kernels for decode-sized batches).

The kernel multiplies the e4m3 values themselves and applies the fp32 block scales to fp32
partial sums, so it differs from the oracle only in summation order; the bound is set by the
re-quantisation of the SiLU*mul output to e4m3 (3 mantissa bits), where a last-bit difference
can flip one element by an e4m3 ulp (up to 12.5 % of that element)."""
import numpy as np
import pytest
import torch

from kernelswift_competition_submission_b200 import (check_device_status, fused_moe, fused_moe_fp8, grouped_topk,
                                                     quantize_rows_fp8, quantize_weights_fp8, softmax_topk)
from oracle.fp8 import moe_experts_fp8_ref, quantize_blocks_128, quantize_rows_128
from torch_ref import experts_rows_fp8

pytestmark = pytest.mark.gpu
TOL8 = 5e-2


FMTS = ["fp32", "ue8m0"]


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("M,K,dtype", [(1, 128, torch.bfloat16), (37, 512, torch.bfloat16), (64, 7168, torch.bfloat16),
                                       (9, 256, torch.float32), (5, 384, torch.float16)])
def test_quantize_rows_bit_exact(cuda_device, M, K, dtype, fmt):
    gen = torch.Generator().manual_seed(M * K)
    x = (torch.randn(M, K, generator=gen) * torch.logspace(-3, 2, M)[:, None]).to(dtype)
    x[0, :128] = 0  # an all-zero block keeps scale 1
    q, s = quantize_rows_fp8(x.to(cuda_device), scale_format=fmt)
    rq, rs = quantize_rows_128(x.float().numpy(), pow2=fmt == "ue8m0")
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    np.testing.assert_array_equal(q.float().cpu().numpy(), rq)


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("E,R,C", [(1, 128, 128), (3, 256, 384), (2, 512, 1024)])
def test_quantize_weights_bit_exact(cuda_device, E, R, C, fmt):
    gen = torch.Generator().manual_seed(E + R + C)
    w = (torch.randn(E, R, C, generator=gen) / C ** 0.5).to(torch.bfloat16)
    q, s = quantize_weights_fp8(w.to(cuda_device), scale_format=fmt)
    rq, rs = quantize_blocks_128(w.float().numpy(), pow2=fmt == "ue8m0")
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    np.testing.assert_array_equal(q.float().cpu().numpy(), rq)


def _fp8_weights(E, K, N, dev, seed, fmt="ue8m0"):
    gen = torch.Generator(device=dev).manual_seed(seed)
    w1 = (torch.randn(E, 2 * N, K, generator=gen, device=dev) / K ** 0.5).to(torch.bfloat16)
    w2 = (torch.randn(E, K, N, generator=gen, device=dev) / N ** 0.5).to(torch.bfloat16)
    w1q, w1s = quantize_weights_fp8(w1, scale_format=fmt)
    w2q, w2s = quantize_weights_fp8(w2, scale_format=fmt)
    return w1q, w1s, w2q, w2s


# (M, E, k): 1 and 37 take the decode kernels (at most 16 pairs per expert), 300, 129 and
# 1024 the prefill GEMMs (block-scaled with ue8m0); 1024 x 4 over 16 experts fills whole
# m-blocks and runs several tiles per CTA
@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("M,E,k,K,N", [(1, 8, 2, 256, 128), (37, 16, 4, 512, 256), (300, 8, 2, 384, 128),
                                       (129, 4, 1, 256, 384), (1024, 16, 4, 1024, 512)])
def test_fused_fp8_oracle(cuda_device, M, E, k, K, N, fmt):
    dev = cuda_device
    w1q, w1s, w2q, w2s = _fp8_weights(E, K, N, dev, seed=M + E, fmt=fmt)
    gen = torch.Generator(device=dev).manual_seed(M)
    x = torch.randn(M, K, generator=gen, device=dev).to(torch.bfloat16)
    w, ids = softmax_topk(torch.randn(M, E, generator=gen, device=dev), k)
    out = fused_moe_fp8(x, w1q, w1s, w2q, w2s, w, ids)
    args = (x.float().cpu().numpy(), w1q.float().cpu().numpy(), w1s.cpu().numpy(), w2q.float().cpu().numpy(),
            w2s.cpu().numpy(), w.cpu().numpy(), ids.cpu().numpy())
    got = out.float().cpu().numpy()
    exact = moe_experts_fp8_ref(*args, pow2=fmt == "ue8m0")
    np.testing.assert_allclose(got, exact, atol=TOL8, rtol=TOL8)
    rel = np.linalg.norm(got - exact) / np.linalg.norm(exact)
    assert rel < 1e-2, rel
    check_device_status(dev)


def test_functional_flag_routes_to_fp8(cuda_device):
    dev = cuda_device
    w1q, w1s, w2q, w2s = _fp8_weights(8, 256, 128, dev, seed=3)
    x = torch.randn(20, 256, device=dev).to(torch.bfloat16)
    w, ids = softmax_topk(torch.randn(20, 8, device=dev), 2)
    a = fused_moe(x, w1q, w2q, w, ids, use_fp8_w8a8=True, w1_scale=w1s, w2_scale=w2s)
    b = fused_moe_fp8(x, w1q, w1s, w2q, w2s, w, ids)
    assert torch.equal(a, b)


@pytest.mark.parametrize("M", [1, 8, 32, 128, 4096])
def test_dsv3_fp8_config(cuda_device, M, dsv3_fp8_weights):
    """DeepSeek-V3 FP8 layer: grouped_topk (sigmoid + bias, top-2 group sum, x2.5) feeding the FP8 expert path."""
    dev = cuda_device
    w1q, w1s, w2q, w2s = dsv3_fp8_weights
    gen = torch.Generator(device=dev).manual_seed(200 + M)
    x = torch.randn(M, 7168, generator=gen, device=dev).to(torch.bfloat16)
    g = torch.randn(M, 256, generator=gen, device=dev)
    bias = torch.randn(256, generator=gen, device=dev) * 0.01
    w, ids = grouped_topk(x, g, 8, True, 8, 4, "sigmoid", 2.5, e_score_correction_bias=bias)
    out = fused_moe_fp8(x, w1q, w1s, w2q, w2s, w, ids)
    rows = torch.randperm(M, generator=gen, device=dev)[:8].cpu()
    ref = experts_rows_fp8(x, w1q, w1s, w2q, w2s, w, ids, rows)
    torch.testing.assert_close(out[rows.to(dev)].float(), ref, atol=TOL8, rtol=TOL8)
    check_device_status(dev)


def test_dsv3_fp8_bench_workload(cuda_device, dsv3_fp8_weights):
    """The FP8 bench workload itself: DeepSeek-V3 layer, 32768 tokens, e4m3 weights with
    128 x 128 block scales. 512 sampled rows (every expert hit) against the fp32
    restatement on the exact dequantised operands: elementwise 5e-2, and the aggregate
    relative error below 2e-2 (at K = 7168 the fp32 sums of GEMM1 differ from the
    restatement's in the last bits, and each such difference that crosses an e4m3
    rounding boundary of the re-quantised SiLU*mul output moves that element by one
    e4m3 step, 6-12 %; about 1.5 % in aggregate here against under 1 % at K <= 512)."""
    dev = cuda_device
    w1q, w1s, w2q, w2s = dsv3_fp8_weights
    M = 32768
    gen = torch.Generator(device=dev).manual_seed(1001)
    x = torch.randn(M, 7168, generator=gen, device=dev).to(torch.bfloat16)
    g = torch.randn(M, 256, generator=gen, device=dev)
    bias = torch.randn(256, generator=torch.Generator(device=dev).manual_seed(44), device=dev) * 0.01
    w, ids = grouped_topk(x, g, 8, True, 8, 4, "sigmoid", 2.5, e_score_correction_bias=bias)
    out = fused_moe(x, w1q, w2q, w, ids, use_fp8_w8a8=True, w1_scale=w1s, w2_scale=w2s)
    torch.cuda.synchronize()
    check_device_status(dev)
    rows = torch.randperm(M, generator=gen, device=dev)[:512].cpu()
    assert torch.unique(ids[rows.to(dev)]).numel() == 256
    ref = experts_rows_fp8(x, w1q, w1s, w2q, w2s, w, ids, rows)
    got = out[rows.to(dev)].float()
    torch.testing.assert_close(got, ref, atol=TOL8, rtol=TOL8)
    assert float((got - ref).norm() / ref.norm()) < 2e-2
    assert torch.isfinite(out).all()


@pytest.fixture(scope="module", params=FMTS)
def dsv3_fp8_weights(cuda_device, request):
    w = _fp8_weights(256, 7168, 2048, cuda_device, seed=43, fmt=request.param)
    torch.cuda.empty_cache()
    yield w
    del w
    torch.cuda.empty_cache()


@pytest.mark.parametrize("M,K", [(1, 128), (37, 512), (64, 7168)])
def test_packed_rows_match_quantize_rows(cuda_device, M, K):
    """Packed e4m3 rows (the expert-parallel FP8 payload) hold the same codes and scales as
    quantize_rows_fp8: K code bytes, then K / 128 fp32 scales."""
    from kernelswift_competition_submission_b200 import fp8_row_bytes, quantize_rows_fp8_packed

    gen = torch.Generator().manual_seed(K + M)
    x = (torch.randn(M, K, generator=gen) * torch.logspace(-2, 1, M)[:, None]).to(torch.bfloat16).to(cuda_device)
    rows = quantize_rows_fp8_packed(x)
    rb = fp8_row_bytes(K)
    assert rows.shape == (M, rb) and rb % 16 == 0 and rb >= K + K // 32
    q, s = quantize_rows_fp8(x)
    assert torch.equal(rows[:, :K], q.view(torch.uint8))
    assert torch.equal(rows[:, K:K + K // 32].contiguous().view(torch.float32), s)


@pytest.mark.parametrize("M,E,k,K,N,pad", [(1, 8, 2, 256, 128, 0), (37, 16, 4, 512, 256, 48),
                                           (300, 8, 2, 384, 128, 16)])
def test_fp8_rows_path_equals_fused_fp8(cuda_device, M, E, k, K, N, pad):
    """The expert path started from packed rows (any 16-byte multiple pitch, -1 slots skipped)
    gives the same bits as fused_moe_fp8 on the tokens those rows came from."""
    from kernelswift_competition_submission_b200 import fp8_row_bytes, fused_moe_fp8_rows, quantize_rows_fp8_packed

    dev = cuda_device
    w1q, w1s, w2q, w2s = _fp8_weights(E, K, N, dev, seed=7 * M + E)
    gen = torch.Generator(device=dev).manual_seed(M + 1)
    x = torch.randn(M, K, generator=gen, device=dev).to(torch.bfloat16)
    w, ids = softmax_topk(torch.randn(M, E, generator=gen, device=dev), k)
    ids = ids.to(torch.int32)
    ids[::5, -1] = -1  # a skipped slot on every fifth token
    rb = fp8_row_bytes(K)
    buf = torch.zeros(M, rb + pad, dtype=torch.uint8, device=dev)
    buf[:, :rb] = quantize_rows_fp8_packed(x)
    got = fused_moe_fp8_rows(buf, K, w1q, w1s, w2q, w2s, w, ids)
    want = fused_moe_fp8(x, w1q, w1s, w2q, w2s, w, ids)
    torch.cuda.synchronize()
    check_device_status(dev)
    assert torch.equal(got, want)
