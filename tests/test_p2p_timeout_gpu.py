"""GPU, one device: a peer-memory wait whose flag nothing sets gives up after its time
limit, records MOE_ERR_TIMEOUT in the status word and leaves the context usable."""
import ctypes
import time

import pytest
import torch

from kernelswift_competition_submission_b200 import _lib, grouped_topk
from kernelswift_competition_submission_b200.ops import _ptr, _stream

pytestmark = pytest.mark.gpu


def test_unset_flag_times_out_with_status(cuda_device):
    lib = _lib.load()
    world, cap, K, k = 1, 4, 64, 2
    base = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    _lib.check(lib.moe_p2p_alloc(world, cap, K, k, ctypes.cast(ctypes.pointer(base), ctypes.c_void_p), handle),
               "alloc")
    try:
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        torch.cuda.synchronize()
        t0 = time.time()
        # the disp flags are 0 and nothing will raise them to 7
        _lib.check(lib.moe_p2p_wait(base, world, 1, cap, K, k, 7, _ptr(status), _stream(cuda_device)), "wait")
        torch.cuda.synchronize()
        waited = time.time() - t0
        assert int(status.item()) == _lib.MOE_ERR_TIMEOUT
        assert 1.0 < waited < 30.0
        # the context still works
        g = torch.randn(16, 256, device=cuda_device)
        w, ids = grouped_topk(None, g, 8, True, 8, 4, "softmax", 1.0)
        torch.cuda.synchronize()
        assert ids.shape == (16, 8)
    finally:
        torch.cuda.synchronize()
        lib.moe_p2p_free(base)
