"""CPU checks of the FP8 oracle (oracle/fp8.py): its e4m3 rounding against PyTorch's own
float8_e4m3fn conversion, and the two scale rules (fp32 amax / 448, and UE8M0: the next
power of two at or above it)."""
import numpy as np
import pytest
import torch

from oracle.fp8 import _scale, dequant_rows, e4m3_round, quantize_blocks_128, quantize_rows_128


def test_e4m3_round_matches_torch_cast():
    rng = np.random.default_rng(5)
    v = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-3, 0.1, 1.0, 30.0, 300.0)])
    v = np.concatenate([v, np.float32([0.0, -0.0, 448.0, -448.0, 2.0 ** -9, 2.0 ** -10, 464.0])])
    ref = torch.from_numpy(np.clip(v, -448, 448)).to(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(e4m3_round(v), ref)


def test_pow2_scale_rule():
    amax = np.float32([0.0, 1e-30, 1e-3, 0.5, 224.0, 448.0, 448.5, 896.0, 3.0e5])
    s = _scale(amax, pow2=True)
    bits = s.view(np.uint32)
    assert np.all(bits & 0x7FFFFF == 0)                      # powers of two
    assert s[0] == 1.0                                          # all-zero block
    lin = _scale(amax)
    assert np.all(s >= lin) and np.all(s[1:] < 2 * lin[1:])     # the next power of two at or above amax / 448
    assert s[5] == 1.0 and s[6] == 2.0 and s[7] == 2.0


@pytest.mark.parametrize("pow2", [False, True])
def test_quantisers_stay_in_range(pow2):
    rng = np.random.default_rng(7)
    x = (rng.standard_normal((6, 512)) * np.logspace(-3, 3, 6)[:, None]).astype(np.float32)
    q, s = quantize_rows_128(x, pow2)
    assert np.abs(q).max() <= 448.0
    rel = np.abs(dequant_rows(q, s) - x).max() / np.abs(x).max()
    assert rel < 2 ** -4
    w = rng.standard_normal((2, 256, 384)).astype(np.float32)
    wq, ws = quantize_blocks_128(w, pow2)
    assert ws.shape == (2, 2, 3) and np.abs(wq).max() <= 448.0
    if pow2:
        assert np.all(ws.view(np.uint32) & 0x7FFFFF == 0)
