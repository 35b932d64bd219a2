"""GPU, one device: the expert-parallel layer over the peer-memory transport after a
bounded wait gave up.

One rank over a one-rank NCCL group runs the layer with ``transport="p2p"`` and then
has a wait on a flag that nothing sets give up after its 2 s limit (no GPU fault: the
kernel returns and records MOE_ERR_TIMEOUT in the status word). From then on the layer
must never hand back stale rows: the next step's kernels do nothing and its output is
NaN, ``check_transport()`` raises, every further forward raises until
``reset_transport()``, and after the reset (new arenas) the layer gives the same bits
as before the failure. The peer-memory kernels run on plain device memory mapped by CUDA
IPC, with no NVLink multicast object.

Also: a freshly allocated arena (``moe_p2p_alloc``) has zeroed flags and counts and -1
in every id row, even when the arena is smaller than 1 KiB.
"""
import ctypes
import os
import socket
import time
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(port, q):
    try:
        from datetime import timedelta

        import torch.distributed as dist

        import kernelswift_competition_submission_b200 as pkg
        from kernelswift_competition_submission_b200 import _lib
        from kernelswift_competition_submission_b200.ep import ExpertParallelMoE
        from kernelswift_competition_submission_b200.ops import _ptr, _stream, status_word

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev, timeout=timedelta(seconds=60))
        E, k, K, N, M = 16, 4, 256, 128, 64
        gen = torch.Generator(device=dev).manual_seed(9)
        w1 = (torch.randn(E, 2 * N, K, generator=gen, device=dev) / K ** 0.5).to(torch.bfloat16)
        w2 = (torch.randn(E, K, N, generator=gen, device=dev) / N ** 0.5).to(torch.bfloat16)
        x = torch.randn(M, K, generator=gen, device=dev).to(torch.bfloat16)
        g = torch.randn(M, E, generator=gen, device=dev)
        layer = ExpertParallelMoE(w1, w2, num_experts=E, topk=k, num_expert_group=4, topk_group=2,
                                  scoring_func="softmax", transport="p2p", max_tokens=M)
        good = layer.forward(x, g)
        layer.check_transport()
        ref = pkg.moe_layer(x, g, w1, w2, topk=k, renormalize=True, num_expert_group=4, topk_group=2)
        torch.cuda.synchronize()
        assert torch.equal(good, ref)
        # a peer that never answers: wait for a disp flag value nothing will write
        p = layer._p2p[0]
        lib = _lib.load()
        st = _stream(dev)
        _lib.check(lib.moe_p2p_wait(ctypes.c_void_p(p["base"]), 1, 1, p["cap"], K, k, p["seq"] + 1000,
                                    _ptr(status_word(dev)), st), "moe_p2p_wait")
        torch.cuda.synchronize()
        assert int(status_word(dev).item()) == _lib.MOE_ERR_TIMEOUT
        t0 = time.time()
        bad = layer.forward(x, g)  # inert kernels: no wait of 2 s each, NaN rows, no stale data
        torch.cuda.synchronize()
        inert_s = time.time() - t0
        assert torch.isnan(bad.float()).all(), "a failed step must not return rows"
        assert inert_s < 1.5, inert_s
        raised = 0
        for call in (layer.check_transport, lambda: layer.forward(x, g)):
            try:
                call()
            except RuntimeError as e:
                assert "reset_transport" in str(e)
                raised += 1
        assert raised == 2
        layer.reset_transport()  # collective; zeroes the status word, new arenas next forward
        again = layer.forward(x, g)
        layer.check_transport()
        torch.cuda.synchronize()
        assert torch.equal(again, ref)
        layer.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put(("ok", ""))
    except Exception:
        q.put(("error", traceback.format_exc()))


def test_p2p_layer_after_timeout_raises_then_recovers(cuda_device):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    proc = ctx.Process(target=_worker, args=(_free_port(), q))
    proc.start()
    res = None
    t0 = time.time()
    while res is None and time.time() - t0 < 180:
        try:
            res = q.get(timeout=2)
        except Exception:
            if not proc.is_alive():
                break
    proc.join(timeout=30)
    if proc.is_alive():
        proc.kill()
    assert res is not None and res[0] == "ok", res


@pytest.mark.parametrize("world,cap,K,k", [(1, 4, 64, 2), (2, 3, 64, 2), (8, 16, 128, 8)])
def test_new_arena_contents(cuda_device, world, cap, K, k):
    from kernelswift_competition_submission_b200 import _lib

    lib = _lib.load()
    base = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    _lib.check(lib.moe_p2p_alloc(world, cap, K, k, ctypes.cast(ctypes.pointer(base), ctypes.c_void_p), handle),
               "moe_p2p_alloc")
    try:
        offs = (ctypes.c_int64 * 9)()
        _lib.check(lib.moe_p2p_arena_offsets(world, cap, K, k, offs), "offsets")
        total = offs[8]
        from cuda.bindings import runtime as rt

        host = torch.empty(total, dtype=torch.uint8)
        (err,) = rt.cudaMemcpy(host.data_ptr(), base.value, total, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
        assert err == rt.cudaError_t.cudaSuccess
        ctrl = host[: offs[4]]
        assert int(ctrl.count_nonzero()) == 0, "flags and counts start at zero"
        ids = host[offs[5]: offs[5] + world * cap * k * 4].view(torch.int32)
        assert bool((ids == -1).all()), "every id row starts empty (-1)"
    finally:
        torch.cuda.synchronize()
        lib.moe_p2p_free(base)
