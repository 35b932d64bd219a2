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
