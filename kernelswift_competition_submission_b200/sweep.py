"""Per-configuration measurements of the MoE-layer path on one B200.

    python -m kernelswift_competition_submission_b200.sweep [--iters N] [--only NAME ...]

One JSON line per configuration row, each timed with CUDA events on the
launching stream after warm-up, L2 flushed (a 256 MiB write) before every
timed call, median over the calls:

  grouped_topk   M = 128 and 32768, E = 256, sigmoid + bias, 8 groups / top-4, k = 8, x2.5
  mixtral        M = 256, E = 8, top-2 softmax routing, K = 4096, N = 14336, bf16
  dsv3_bf16      grouped_topk + fused_moe at the DeepSeek-V3 shape, M = 1, 64, 512, 4096
  dsv3_fp8       the same with e4m3 weights (128 x 128 block scales) and per-token-per-128
                 activation quantisation, M = 1, 8, 32, 128
  tasks          the reference's task shapes through the drop-in ModelNew modules (latency per
                 call, the harness's protocol), graph replay and eager
  router         router GEMM fused with grouped_topk, M = 1, 128, 4096, 32768, against the
                 unfused pair (cuBLAS bf16 GEMM + grouped_topk)
  decode_graph   the DeepSeek-V3 bf16 layer at M = 1, 8, 64, eager and as one replayed CUDA graph
  ep_one_rank    (only when named) the expert-parallel layer over a one-rank NCCL group,
                 M = 16384, bf16 and FP8, NCCL and peer-arena transports: per-phase times of
                 one rank (the same rows reach the expert stage through either transport)

Each line carries the algorithmic work (FLOPs = 6 M k K N for the expert path;
bytes = A 3 K N b_w (+ block scales) + M K b_x + M K 2 + M k 8 + M E 4 with A the
distinct experts hit; grouped_topk alone: M E 4 + E 4 + M k 8), the binding
roofline (measured HBM GB/s or tensor TFLOP/s from MEASURED_PEAKS.json, e4m3 at
twice the bf16 rate) and the fraction of it achieved. Inputs are seeded synthetic
Gaussians with the configurations' shapes; weights ~N(0, 1/sqrt(fan_in)).
"""

from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

import torch

from . import ops

ROOT = Path(__file__).resolve().parent.parent


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class _Timer:
    def __init__(self, dev):
        self.flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def median_ms(self, fn, iters: int, warmup: int = 3) -> float:
        for _ in range(warmup):
            fn()
        ts = []
        for _ in range(iters):
            self.flush.fill_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts)


def _weights(E, K, N, dev, seed):
    w1 = torch.empty(E, 2 * N, K, dtype=torch.bfloat16, device=dev)
    w2 = torch.empty(E, K, N, dtype=torch.bfloat16, device=dev)
    for e in range(E):
        g = torch.Generator(device=dev).manual_seed(seed + e)
        w1[e].copy_(torch.randn(2 * N, K, generator=g, device=dev) / K ** 0.5)
        w2[e].copy_(torch.randn(K, N, generator=g, device=dev) / N ** 0.5)
    return w1, w2


def _line(name, M, ms, flops, nbytes, peaks, tc_tflops, extra=None):
    t_tc = flops / (tc_tflops * 1e12) if flops else 0.0
    t_hbm = nbytes / (peaks["hbm_gbs"] * 1e9)
    bound = "tensor" if t_tc > t_hbm else "hbm"
    d = {"config": name, "tokens": M, "ms": ms, "tokens_per_s": M / (ms / 1e3),
         "tflops": flops / (ms / 1e3) / 1e12 if flops else None, "gbs": nbytes / (ms / 1e3) / 1e9,
         "alg_flops": flops, "alg_bytes": nbytes, "bound": bound,
         "roofline_frac": max(t_tc, t_hbm) / (ms / 1e3),
         "peak": {"hbm_gbs": peaks["hbm_gbs"], "tensor_tflops": tc_tflops, "source": peaks["source"]}}
    if extra:
        d.update(extra)
    print(json.dumps(d), flush=True)


def sweep_grouped_topk(dev, timer, peaks, iters):
    E, k = 256, 8
    bias = torch.randn(E, generator=torch.Generator(device=dev).manual_seed(44), device=dev) * 0.01
    for M in (128, 32768):
        g = torch.randn(M, E, generator=torch.Generator(device=dev).manual_seed(M), device=dev)
        x = torch.empty(M, 1, dtype=torch.bfloat16, device=dev)
        ms = timer.median_ms(lambda: ops.grouped_topk(x, g, k, True, 8, 4, "sigmoid", 2.5,
                                                      e_score_correction_bias=bias), iters)
        _line("grouped_topk", M, ms, 0, M * E * 4 + E * 4 + M * k * 8, peaks, peaks["bf16_tflops"])


def _layer_bytes(ids, E, K, N, M, k, wbytes, scale_bytes=0):
    A = int(torch.unique(ids).numel())
    return A * (3 * K * N * wbytes + scale_bytes) + M * K * 2 * 2 + M * k * 8 + M * E * 4, A


def sweep_mixtral(dev, timer, peaks, iters):
    E, k, K, N, M = 8, 2, 4096, 14336, 256
    w1, w2 = _weights(E, K, N, dev, seed=5000)
    gen = torch.Generator(device=dev).manual_seed(42)
    x = torch.randn(M, K, generator=gen, device=dev).to(torch.bfloat16)
    logits = torch.randn(M, E, generator=gen, device=dev)
    out = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(ops.fused_moe_workspace_bytes(M, E, k, K, N), dtype=torch.uint8, device=dev)

    def run():
        w, ids = ops.softmax_topk(logits, k)
        ops.fused_moe(x, w1, w2, w, ids, out=out, workspace=ws)

    ms = timer.median_ms(run, iters)
    _, ids = ops.softmax_topk(logits, k)
    nbytes, A = _layer_bytes(ids, E, K, N, M, k, 2)
    _line("mixtral_bf16", M, ms, 6.0 * M * k * K * N, nbytes, peaks, peaks["bf16_tflops"], {"experts_hit": A})


def _dsv3_inputs(M, dev):
    gen = torch.Generator(device=dev).manual_seed(1000 + M)
    x = torch.randn(M, 7168, generator=gen, device=dev).to(torch.bfloat16)
    g = torch.randn(M, 256, generator=gen, device=dev)
    bias = torch.randn(256, generator=torch.Generator(device=dev).manual_seed(44), device=dev) * 0.01
    return x, g, bias


def sweep_dsv3(dev, timer, peaks, iters, fp8: bool):
    E, k, K, N = 256, 8, 7168, 2048
    w1, w2 = _weights(E, K, N, dev, seed=43_000)
    if fp8:
        w1q, w1s = ops.quantize_weights_fp8(w1)
        w2q, w2s = ops.quantize_weights_fp8(w2)
        del w1, w2
        torch.cuda.empty_cache()
    for M in ((1, 8, 32, 128) if fp8 else (1, 64, 512, 4096)):
        x, g, bias = _dsv3_inputs(M, dev)
        out = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
        if fp8:
            ws = torch.empty(int(ops._lib.load().moe_fused_workspace_bytes_fp8(M, E, k, K, N)), dtype=torch.uint8,
                             device=dev)
        else:
            ws = torch.empty(ops.fused_moe_workspace_bytes(M, E, k, K, N), dtype=torch.uint8, device=dev)

        def run():
            w, ids = ops.grouped_topk(x, g, k, True, 8, 4, "sigmoid", 2.5, e_score_correction_bias=bias)
            if fp8:
                ops.fused_moe_fp8(x, w1q, w1s, w2q, w2s, w, ids, out=out, workspace=ws)
            else:
                ops.fused_moe(x, w1, w2, w, ids, out=out, workspace=ws)

        ms = timer.median_ms(run, iters)
        _, ids = ops.grouped_topk(x, g, k, True, 8, 4, "sigmoid", 2.5, e_score_correction_bias=bias)
        scale_bytes = 3 * (K // 128) * (N // 128) * 4 if fp8 else 0
        nbytes, A = _layer_bytes(ids, E, K, N, M, k, 1 if fp8 else 2, scale_bytes)
        tc = peaks["bf16_tflops"] * (2.0 if fp8 else 1.0)
        _line("dsv3_fp8" if fp8 else "dsv3_bf16", M, ms, 6.0 * M * k * K * N, nbytes, peaks, tc,
              {"experts_hit": A})
        ops.check_device_status(dev)


def sweep_decode_graph(dev, timer, peaks, iters):
    """DeepSeek-V3 bf16 layer (grouped_topk + fused_moe) at decode sizes, each call eager
    (one launch per kernel, host work between) and replayed as one CUDA graph of the whole
    layer (graphs.GraphCache on the same buffers)."""
    from .graphs import GraphCache

    E, k, K, N = 256, 8, 7168, 2048
    w1, w2 = _weights(E, K, N, dev, seed=43_000)
    for M in (1, 8, 64):
        x, g, bias = _dsv3_inputs(M, dev)

        def layer(xx, gg):
            return ops.moe_layer(xx, gg, w1, w2, topk=k, renormalize=True, num_expert_group=8, topk_group=4,
                                 scoring_func="sigmoid", routed_scaling_factor=2.5, e_score_correction_bias=bias)

        eager = timer.median_ms(lambda: layer(x, g), iters)
        cache = GraphCache(layer)
        graph = timer.median_ms(lambda: cache(x, g), iters)
        _, ids = ops.grouped_topk(x, g, k, True, 8, 4, "sigmoid", 2.5, e_score_correction_bias=bias)
        nbytes, A = _layer_bytes(ids, E, K, N, M, k, 2)
        _line("dsv3_bf16_graph", M, graph, 6.0 * M * k * K * N, nbytes, peaks, peaks["bf16_tflops"],
              {"experts_hit": A, "eager_ms": eager, "replays": cache.replays})


def sweep_ep_one_rank(dev, iters):
    """ExpertParallelMoE over a one-rank NCCL group at the DeepSeek-V3 shape, M = 16384: mean
    per-phase CUDA-event times over `iters` forwards after 3 warm-ups, for bf16 and FP8
    weights and both transports."""
    import os
    import socket

    import torch.distributed as dist

    from .ep import ExpertParallelMoE

    if not dist.is_initialized():
        with socket.socket() as sk:
            sk.bind(("127.0.0.1", 0))
            port = sk.getsockname()[1]
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(port))
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=dev)
    E, k, K, N, M = 256, 8, 7168, 2048, 16384
    x, g, bias = _dsv3_inputs(M, dev)
    for fp8 in (False, True):
        w1, w2 = _weights(E, K, N, dev, seed=43_000)
        kw = {}
        if fp8:
            w1, s1 = ops.quantize_weights_fp8(w1)
            w2, s2 = ops.quantize_weights_fp8(w2)
            kw = dict(use_fp8_w8a8=True, w1_scale=s1, w2_scale=s2)
        torch.cuda.empty_cache()
        for transport in ("nccl", "p2p"):
            layer = ExpertParallelMoE(w1, w2, num_experts=E, topk=k, num_expert_group=8, topk_group=4,
                                      scoring_func="sigmoid", routed_scaling_factor=2.5,
                                      e_score_correction_bias=bias, transport=transport, chunks=1, **kw)
            for _ in range(3):
                layer.forward(x, g)
            torch.cuda.synchronize()
            layer.profile, layer.phase_log = True, []
            for _ in range(iters):
                layer.forward(x, g)
            layer.profile = False
            ph = layer.phase_breakdown()
            print(json.dumps({"config": "ep_one_rank", "M": M, "dtype": "fp8" if fp8 else "bf16",
                              "transport": transport, "ms_per_step": sum(ph.values()),
                              "phases_ms": {n: round(v, 4) for n, v in ph.items()}}), flush=True)
            layer.close()
            ops.check_device_status(dev)
        del w1, w2
        torch.cuda.empty_cache()
    dist.destroy_process_group()


def sweep_tasks(dev, iters_unused=None):
    """The reference's own task shapes through the drop-in ModelNew modules, timed the way
    its harness times them: per call, host clock around the call and a device synchronise,
    200 warm-up calls, median of 500. Reported for the graph-replay forward and for the
    eager forward (the same ops launched one by one)."""
    import importlib.util
    import time

    tasks = Path(__file__).resolve().parent / "tasks"

    def load(name):
        spec = importlib.util.spec_from_file_location(f"task_{name}", tasks / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod

    def median_call_ms(fn, args):
        for _ in range(200):
            fn(*args)
        torch.cuda.synchronize()
        ts = []
        for _ in range(500):
            t0 = time.perf_counter()
            fn(*args)
            torch.cuda.synchronize()
            ts.append((time.perf_counter() - t0) * 1e3)
        return statistics.median(ts)

    torch.manual_seed(42)
    for name in ("grouped_topk", "fused_moe"):
        mod = load(name)
        model = mod.ModelNew(*mod.get_init_inputs()).to(dev)
        args = [t.to(dev) for t in mod.get_inputs()]
        with torch.no_grad():
            graph_ms = median_call_ms(model, args)
            if name == "fused_moe":
                w1, w2 = model._prepared_weights(args[0].dtype)
                eager_ms = median_call_ms(lambda a, b: model._forward_eager(a, b, w1, w2), args)
            else:
                eager_ms = median_call_ms(model._forward_eager, args)
        print(json.dumps({"config": f"task_{name}", "tokens": int(args[0].shape[0]), "graph_replay_ms": graph_ms,
                          "eager_ms": eager_ms, "protocol": "host clock per call + synchronize, median of 500 "
                                                            "after 200 warm-up calls"}), flush=True)


def sweep_router(dev, timer, peaks, iters):
    """Router GEMM fused with grouped_topk (E = 256, K = 7168, sigmoid + bias, 8 groups / top-4,
    k = 8) against the same two steps unfused: the bf16 GEMM by torch (cuBLAS) and the
    grouped_topk kernel on its (fp32-cast) output."""
    E, K, k = 256, 7168, 8
    wg = (torch.randn(E, K, generator=torch.Generator(device=dev).manual_seed(7), device=dev) / K ** 0.5).bfloat16()
    bias = torch.randn(E, generator=torch.Generator(device=dev).manual_seed(44), device=dev) * 0.01
    for M in (1, 128, 4096, 32768):
        x = torch.randn(M, K, generator=torch.Generator(device=dev).manual_seed(M), device=dev).bfloat16()
        fused = timer.median_ms(lambda: ops.router_grouped_topk(x, wg, k, True, 8, 4, "sigmoid", 2.5,
                                                                e_score_correction_bias=bias), iters)
        unfused = timer.median_ms(lambda: ops.grouped_topk(x, (x @ wg.T).float(), k, True, 8, 4, "sigmoid", 2.5,
                                                           e_score_correction_bias=bias), iters)
        flops = 2.0 * M * K * E
        nbytes = E * K * 2 + M * K * 2 + M * k * 8
        _line("router_fused", M, fused, flops, nbytes, peaks, peaks["bf16_tflops"], {"unfused_ms": unfused})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", nargs="*", default=None,
                    choices=["grouped_topk", "mixtral", "dsv3_bf16", "dsv3_fp8", "tasks", "router",
                             "decode_graph", "ep_one_rank"])
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks = _peaks()
    timer = _Timer(dev)
    want = set(a.only or ["grouped_topk", "mixtral", "dsv3_bf16", "dsv3_fp8", "tasks", "router", "decode_graph"])
    if "decode_graph" in want:
        sweep_decode_graph(dev, timer, peaks, a.iters)
        torch.cuda.empty_cache()
    if "router" in want:
        sweep_router(dev, timer, peaks, a.iters)
    if "tasks" in want:
        sweep_tasks(dev)
    if "grouped_topk" in want:
        sweep_grouped_topk(dev, timer, peaks, a.iters)
    if "mixtral" in want:
        sweep_mixtral(dev, timer, peaks, a.iters)
        torch.cuda.empty_cache()
    if "dsv3_bf16" in want:
        sweep_dsv3(dev, timer, peaks, a.iters, fp8=False)
        torch.cuda.empty_cache()
    if "dsv3_fp8" in want:
        sweep_dsv3(dev, timer, peaks, a.iters, fp8=True)
    if "ep_one_rank" in want:  # named only: it sets up a one-rank process group
        sweep_ep_one_rank(dev, a.iters)


if __name__ == "__main__":
    main()
