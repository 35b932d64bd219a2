"""CPU: the expert-parallel dispatch / combine logic on gloo ranks (world size 2 and 4).

The layer's routing and expert stages are replaced by the numpy oracle, so
these tests exercise exactly the host-side plan, the all-to-all exchanges and
the combine of ``ExpertParallelMoE``; its output must equal the single-process
oracle layer on the same tokens. A second test makes one rank leave before a
collective and checks that the others fail with an error instead of hanging.
"""
import os
import socket
import time
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kernelswift_competition_submission_b200.ep import ExpertParallelMoE, plan_dispatch
from oracle.fused_moe import moe_experts_ref
from oracle.grouped_topk import grouped_topk_ref

E, K_TOP, HID, INTER, NG, TG = 16, 4, 32, 16, 4, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights():
    rng = np.random.default_rng(123)
    w1 = rng.standard_normal((E, 2 * INTER, HID), dtype=np.float32) / np.sqrt(HID)
    w2 = rng.standard_normal((E, HID, INTER), dtype=np.float32) / np.sqrt(INTER)
    return w1, w2


def _tokens(rank, m):
    rng = np.random.default_rng(1000 + rank)
    return rng.standard_normal((m, HID), dtype=np.float32), rng.standard_normal((m, E), dtype=np.float32)


def _route(x, g):
    w, ids = grouped_topk_ref(g.numpy(), K_TOP, True, NG, TG, "sigmoid", 2.5,
                              np.linspace(-0.01, 0.01, E, dtype=np.float32), "top2sum")
    return torch.from_numpy(w), torch.from_numpy(ids)


def _worker(rank, world, port, q, m_per_rank):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
        w1, w2 = _weights()
        el = E // world
        w1l, w2l = w1[rank * el:(rank + 1) * el], w2[rank * el:(rank + 1) * el]

        def experts(x, w, ids, events=None):
            ids_np = ids.numpy()
            w_np = np.where(ids_np >= 0, w.numpy(), 0.0).astype(np.float32)
            if x.shape[0] == 0:
                return torch.zeros(0, HID)
            return torch.from_numpy(moe_experts_ref(x.numpy(), w1l, w2l, w_np, np.clip(ids_np, 0, None)))

        layer = ExpertParallelMoE(torch.from_numpy(w1l), torch.from_numpy(w2l), num_experts=E, topk=K_TOP,
                                  route_fn=_route, expert_fn=experts)
        m = m_per_rank[rank]
        x, g = _tokens(rank, m)
        out = layer.forward(torch.from_numpy(x), torch.from_numpy(g))
        w, ids = _route(None, torch.from_numpy(g))
        ref = moe_experts_ref(x, w1, w2, w.numpy(), ids.numpy())
        err = float(np.abs(out.numpy() - ref).max()) if m else 0.0
        q.put((rank, "ok", err))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def _run(world, m_per_rank, target=_worker, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q, m_per_rank)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    t0 = time.time()
    while len(results) < world and time.time() - t0 < timeout:
        try:
            r, status, val = q.get(timeout=1)
            results[r] = (status, val)
        except Exception:
            if not any(p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("world,m", [(2, [37, 50]), (4, [20, 0, 33, 8])])
def test_ep_matches_single_process(world, m):
    res = _run(world, m)
    assert len(res) == world, res
    for r, (status, val) in res.items():
        assert status == "ok", val
        assert val < 1e-4, f"rank {r} max err {val}"


def test_plan_dispatch_dedups_and_orders():
    ids = torch.tensor([[0, 1, 5, 7], [6, 7, 2, 3], [1, 0, 3, 2]], dtype=torch.int32)
    w = torch.arange(12, dtype=torch.float32).view(3, 4)
    tok, counts, lids, lw = plan_dispatch(ids, w, experts_per_rank=4, world=2)
    assert counts.tolist() == [3, 2]                   # rank 0 gets all 3 tokens, rank 1 gets tokens 0 and 1
    assert tok.tolist() == [0, 1, 2, 0, 1]
    assert lids.tolist()[0] == [0, 1, -1, -1]
    assert lids.tolist()[3] == [-1, -1, 1, 3]
    assert lids.tolist()[4] == [2, 3, -1, -1]
    assert torch.equal(lw[3], w[0])


def _leaver(rank, world, port, q, m_per_rank):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
        if rank == 1:
            q.put((rank, "left", ""))
            q.close()
            q.join_thread()
            os._exit(0)  # leaves between steps, before the next collective
        t0 = time.time()
        counts = torch.ones(world, dtype=torch.int64)
        out = torch.empty_like(counts)
        try:
            dist.all_to_all_single(out, counts)
            q.put((rank, "no-error", time.time() - t0))
        except Exception as e:  # the peer is gone: the collective must fail, not hang
            q.put((rank, "raised", f"{type(e).__name__} after {time.time() - t0:.1f}s"))
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def test_rank_leaving_makes_peers_fail_not_hang():
    res = _run(2, [0, 0], target=_leaver, timeout=60)
    assert res.get(1, ("?",))[0] == "left", res
    assert res.get(0, ("?",))[0] == "raised", res


def _worker_replicated(rank, world, port, q, m_per_rank):
    """Same as _worker, with the three busiest experts replicated on every rank (weights
    broadcast from their owners by ``rebalance``)."""
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
        w1, w2 = _weights()
        el = E // world
        w1l, w2l = w1[rank * el:(rank + 1) * el], w2[rank * el:(rank + 1) * el]
        holder = {}

        def experts(x, w, ids, events=None):
            lw1, lw2 = holder["layer"].w1.numpy(), holder["layer"].w2.numpy()
            ids_np = ids.numpy()
            w_np = np.where(ids_np >= 0, w.numpy(), 0.0).astype(np.float32)
            if x.shape[0] == 0:
                return torch.zeros(0, HID)
            return torch.from_numpy(moe_experts_ref(x.numpy(), lw1, lw2, w_np, np.clip(ids_np, 0, None)))

        layer = ExpertParallelMoE(torch.from_numpy(w1l), torch.from_numpy(w2l), num_experts=E, topk=K_TOP,
                                  route_fn=_route, expert_fn=experts)
        holder["layer"] = layer
        m = m_per_rank[rank]
        x, g = _tokens(rank, m)
        _, ids = _route(None, torch.from_numpy(g))
        hot = layer.rebalance(ids, 3)  # replica weights broadcast from their owners
        out = layer.forward(torch.from_numpy(x), torch.from_numpy(g))
        w, ids = _route(None, torch.from_numpy(g))
        ref = moe_experts_ref(x, w1, w2, w.numpy(), ids.numpy())
        err = float(np.abs(out.numpy() - ref).max()) if m else 0.0
        q.put((rank, "ok", (err, hot)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("world,m", [(2, [37, 50]), (4, [20, 0, 33, 8])])
def test_ep_replicated_hot_experts_match(world, m):
    res = _run(world, m, target=_worker_replicated)
    assert len(res) == world, res
    hots = set()
    for r, (status, val) in res.items():
        assert status == "ok", val
        err, hot = val
        assert err < 1e-4, f"rank {r} max err {err}"
        hots.add(tuple(hot))
    assert len(hots) == 1  # every rank picked the same experts


def test_plan_dispatch_with_expert_map_keeps_replicas_home():
    # 8 experts on 2 ranks; rank 1's view: expert 2 (owned by rank 0) replicated at rank 1, local slot 4
    emap = torch.tensor([(e // 4) << 16 | (e % 4) for e in range(8)], dtype=torch.int32)
    emap[2] = (1 << 16) | 4
    ids = torch.tensor([[2, 5], [0, 2], [2, 6]], dtype=torch.int32)
    w = torch.ones(3, 2)
    tok, counts, lids, _ = plan_dispatch(ids, w, experts_per_rank=4, world=2, expert_map=emap)
    assert counts.tolist() == [1, 3]                    # only token 1's expert 0 leaves for rank 0
    assert tok.tolist() == [1, 0, 1, 2]
    assert lids.tolist() == [[0, -1], [4, 1], [-1, 4], [4, 2]]


# ---------------------------------------------------------------- FP8 payload (packed e4m3 rows)
HID8, INTER8 = 256, 128


def _pack_rows(x):
    """Packed e4m3 rows as the library lays them out: K codes, then K / 128 fp32 scales
    (padded to 16 bytes), from the oracle's per-token-per-128 quantisation."""
    from oracle.fp8 import quantize_rows_128

    K = x.shape[1]
    if x.shape[0] == 0:
        return torch.zeros(0, K + (K // 32 + 15) // 16 * 16, dtype=torch.uint8)
    q, s = quantize_rows_128(x.numpy())
    codes = torch.from_numpy(q).to(torch.float8_e4m3fn).view(torch.uint8)
    scales = torch.from_numpy(np.ascontiguousarray(s)).view(torch.uint8)
    pad = (-(codes.shape[1] + scales.shape[1])) % 16
    return torch.cat([codes, scales, torch.zeros(x.shape[0], pad, dtype=torch.uint8)], dim=1).contiguous()


def _unpack_rows(rows, K):
    q = rows[:, :K].contiguous().view(torch.float8_e4m3fn).float().numpy()
    s = rows[:, K:K + K // 32].contiguous().view(torch.float32).numpy()
    return q, s


def _worker_fp8(rank, world, port, q, cfg):
    """FP8 layer on gloo ranks: the packed e4m3 rows travel; each rank's expert stage reads
    them back and runs the oracle on its own experts' slots (and, with n_hot > 0, on the
    replicas of the n_hot busiest experts, e4m3 weights and block scales broadcast by
    ``rebalance``)."""
    m_per_rank, n_hot = cfg
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta

        from oracle.fp8 import moe_experts_fp8_ref, moe_experts_fp8_rows_ref, quantize_blocks_128

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
        rng = np.random.default_rng(321)
        w1 = rng.standard_normal((E, 2 * INTER8, HID8), dtype=np.float32) / np.sqrt(HID8)
        w2 = rng.standard_normal((E, HID8, INTER8), dtype=np.float32) / np.sqrt(INTER8)
        w1q, w1s = quantize_blocks_128(w1)
        w2q, w2s = quantize_blocks_128(w2)
        el = E // world
        sl = slice(rank * el, (rank + 1) * el)

        def as_e4m3(a):
            return torch.from_numpy(np.ascontiguousarray(a)).to(torch.float8_e4m3fn)

        holder = {}

        def experts(rows, w, ids, events=None):
            ids_np = ids.numpy()
            if rows.shape[0] == 0:
                return torch.zeros(0, HID8)
            xq, xs = _unpack_rows(rows, HID8)
            w_np = np.where(ids_np >= 0, w.numpy(), 0.0).astype(np.float32)
            lay = holder["layer"]  # the layer's own expert table (replicas appended by rebalance)
            lw1 = lay.w1.view(torch.float8_e4m3fn).float().numpy()
            lw2 = lay.w2.view(torch.float8_e4m3fn).float().numpy()
            return torch.from_numpy(moe_experts_fp8_rows_ref(xq, xs, lw1, lay.w1s.numpy(), lw2, lay.w2s.numpy(),
                                                             w_np, ids_np))

        layer = ExpertParallelMoE(as_e4m3(w1q[sl]), as_e4m3(w2q[sl]), num_experts=E, topk=K_TOP, route_fn=_route,
                                  expert_fn=experts, use_fp8_w8a8=True, w1_scale=torch.from_numpy(w1s[sl].copy()),
                                  w2_scale=torch.from_numpy(w2s[sl].copy()), quant_fn=_pack_rows)
        holder["layer"] = layer
        m = m_per_rank[rank]
        rng_t = np.random.default_rng(2000 + rank)
        x = rng_t.standard_normal((m, HID8), dtype=np.float32)
        g = rng_t.standard_normal((m, E), dtype=np.float32)
        if n_hot:
            _, ids0 = _route(None, torch.from_numpy(g))
            hot = layer.rebalance(ids0, n_hot)
            assert hot == layer.replicated and layer.w1s.shape[0] == el + n_hot
        out = layer.forward(torch.from_numpy(x), torch.from_numpy(g))
        w, ids = _route(None, torch.from_numpy(g))
        ref = moe_experts_fp8_ref(x, w1q, w1s, w2q, w2s, w.numpy(), ids.numpy())
        err = float(np.abs(out.numpy() - ref).max()) if m else 0.0
        q.put((rank, "ok", err))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


@pytest.mark.parametrize("world,m,n_hot", [(2, [37, 50], 0), (4, [20, 0, 33, 8], 0), (4, [25, 40, 0, 12], 3)])
def test_ep_fp8_payload_matches_single_process(world, m, n_hot):
    """The packed e4m3 rows survive pack -> all-to-all -> expert stage unchanged: the layer
    equals the single-process FP8 oracle on the same tokens (fp32 summation order only),
    also with hot experts replicated from their owners' e4m3 weights and scales."""
    res = _run(world, (m, n_hot), target=_worker_fp8)
    assert len(res) == world, res
    for r, (status, val) in res.items():
        assert status == "ok", val
        assert val < 1e-4, f"rank {r} max err {val}"


def _launch_counts(rank, world, port, q, unused):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        from datetime import timedelta

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
        w1, w2 = _weights()
        el = E // world
        w1l, w2l = torch.from_numpy(w1[:el]), torch.from_numpy(w2[:el])
        w8a, w8b = torch.zeros(el, 256, 128, dtype=torch.uint8), torch.zeros(el, 128, 128, dtype=torch.uint8)
        s8a, s8b = torch.ones(el, 2, 1), torch.ones(el, 1, 1)
        got = {}
        for name, kw, a, b in (("nccl1", dict(chunks=1), w1l, w2l), ("nccl2", dict(chunks=2), w1l, w2l),
                               ("p2p", dict(transport="p2p"), w1l, w2l),
                               ("fp8_nccl2", dict(chunks=2, use_fp8_w8a8=True, w1_scale=s8a, w2_scale=s8b), w8a, w8b),
                               ("fp8_p2p", dict(transport="p2p", use_fp8_w8a8=True, w1_scale=s8a, w2_scale=s8b), w8a,
                                w8b)):
            got[name] = ExpertParallelMoE(a, b, num_experts=E, topk=K_TOP, **kw).kernel_launches_per_step
        q.put((rank, "ok", got))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "error", traceback.format_exc()))


def test_kernel_launch_counts_per_transport():
    """The launch count the bench reports follows the forward that runs: routing + 8 kernels
    per token chunk (NCCL, bf16), + quantise once and 2 gathers per chunk (FP8), 11 / 14 kernels
    through the peer arenas."""
    res = _run(2, None, target=_launch_counts)
    assert len(res) == 2, res
    for r, (status, val) in res.items():
        assert status == "ok", val
        assert val == {"nccl1": 9, "nccl2": 17, "p2p": 11, "fp8_nccl2": 22, "fp8_p2p": 14}, val
