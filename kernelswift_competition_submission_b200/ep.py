"""Expert-parallel MoE layer over NCCL (one process per GPU).

The reference has no multi-device code; this layer is the expert-parallel
form of its MoE path (``grouped_topk`` routing feeding ``fused_moe``,
``fused_moe/v0/fused_moe.py:126-167``). Rank r owns the contiguous experts
``[r * E / G, (r + 1) * E / G)`` and its own M / G tokens. One forward:

1. route the rank's tokens with ``grouped_topk`` (sigmoid + bias, top-2 group
   sum for DeepSeek-V3);
2. plan: for each token, the set of ranks owning at least one of its top-k
   experts; the token is sent once per such rank (deduplicated), carrying its
   k weights and its k expert ids rewritten to that rank's local numbering
   (-1 for slots that rank does not own);
3. exchange per-destination row counts (``all_to_all_single``), then the rows
   and the (ids, weights) metadata (``all_to_all_single`` with split sizes);
4. run the local expert path on the received rows (``fused_moe``: -1 ids
   contribute nothing, so each received row comes back as the weighted sum over
   this rank's experts only);
5. send the partial rows back with the reverse splits and sum them per token in
   fp32.

On CUDA tensors steps 2 and 5 are the library's kernels (``moe_ep_plan``,
``moe_ep_pack``, ``moe_ep_combine``); on CPU tensors (the gloo tests) the
same plan is restated with torch ops (``plan_dispatch``).

Collectives go through ``torch.distributed`` (NCCL over NVLink/NVSwitch on
B200; gloo in the CPU tests); no kernel waits on another rank. Every rank takes
the same collective steps in the same order, including for empty splits.

``route_fn`` / ``expert_fn`` default to this package's CUDA ops; the CPU tests
inject the numpy oracle to check the dispatch/combine logic on gloo ranks.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def plan_dispatch(ids: torch.Tensor, w: torch.Tensor, experts_per_rank: int, world: int):
    """Deduplicated per-destination send list for routed tokens.

    ids int [M, k] global expert ids, w float [M, k].
    Returns (send_tok int64 [S], send_counts int64 [world], send_ids int32 [S, k], send_w fp32 [S, k]),
    rows ordered by destination rank then token.
    """
    M, k = ids.shape
    ids64 = ids.long()
    valid = (ids64 >= 0) & (ids64 < experts_per_rank * world)
    dst = torch.div(ids64, experts_per_rank, rounding_mode="floor").clamp(0, world - 1)
    hit = torch.zeros(M, world, dtype=torch.int32, device=ids.device)
    hit.scatter_add_(1, dst, valid.to(torch.int32))
    hit = hit > 0
    send_dst, send_tok = hit.t().nonzero(as_tuple=True)  # sorted by destination, then token
    send_counts = hit.sum(0).to(torch.int64)
    own = (dst[send_tok] == send_dst[:, None]) & valid[send_tok]
    local = ids64[send_tok] - send_dst[:, None] * experts_per_rank
    send_ids = torch.where(own, local, torch.full_like(local, -1)).to(torch.int32)
    send_w = w[send_tok].to(torch.float32)
    return send_tok, send_counts, send_ids, send_w


class ExpertParallelMoE:
    """MoE layer with experts sharded over the ranks of ``group``.

    w1_local [E/G, 2N, K], w2_local [E/G, K, N]: this rank's experts.
    """

    def __init__(self, w1_local, w2_local, *, num_experts, topk, num_expert_group=1, topk_group=1,
                 scoring_func="softmax", routed_scaling_factor=1.0, e_score_correction_bias=None,
                 renormalize=True, group=None, route_fn=None, expert_fn=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"num_experts {num_experts} must divide by the world size {self.world}")
        self.E = num_experts
        self.E_local = num_experts // self.world
        if w1_local.shape[0] != self.E_local or w2_local.shape[0] != self.E_local:
            raise ValueError("w1_local / w2_local must hold num_experts / world experts")
        self.w1, self.w2 = w1_local, w2_local
        self.topk = topk
        self.route_kw = dict(topk=topk, renormalize=renormalize, num_expert_group=num_expert_group,
                             topk_group=topk_group, scoring_func=scoring_func,
                             routed_scaling_factor=routed_scaling_factor,
                             e_score_correction_bias=e_score_correction_bias)
        self.route_fn = route_fn or self._route_cuda
        self.expert_fn = expert_fn or self._experts_cuda
        # routing, EP count, EP pack, align count, align scatter, GEMM1, GEMM2, combine, EP combine
        self.kernel_launches_per_step = 9
        self._ws = None
        # per-phase CUDA events of each forward when `profile` is set (bench breakdown)
        self.profile = False
        self.phase_log = []
        self._on_cuda = False
        self._marks = []

    # ------------------------------------------------------------------ default (CUDA) stages
    def _route_cuda(self, x, gating):
        from .ops import grouped_topk

        kw = self.route_kw
        return grouped_topk(x, gating, kw["topk"], kw["renormalize"], kw["num_expert_group"], kw["topk_group"],
                            kw["scoring_func"], kw["routed_scaling_factor"], kw["e_score_correction_bias"])

    def _experts_cuda(self, x, w, ids, events=None):
        from .ops import fused_moe_staged, fused_moe_workspace_bytes

        M = x.shape[0]
        if M == 0:
            if events:
                for e in events:
                    e.record()
            return torch.empty(0, x.shape[1], dtype=x.dtype, device=x.device)
        need = fused_moe_workspace_bytes(M, self.E_local, ids.shape[1], x.shape[1], self.w2.shape[2])
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(int(need * 1.25) + 256, dtype=torch.uint8, device=x.device)
        return fused_moe_staged(x, self.w1, self.w2, w, ids, workspace=self._ws, events=events)

    # ------------------------------------------------------------------ forward
    def _mark(self, name):
        if self.profile and self._on_cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._marks.append((name, ev))

    def forward(self, x: torch.Tensor, gating: torch.Tensor, events=None) -> torch.Tensor:
        M, K = x.shape
        self._on_cuda = x.is_cuda
        self._marks = []
        self._mark("start")
        w, ids = self.route_fn(x, gating)
        self._mark("route")
        if x.is_cuda:
            send_x, send_meta, send_counts, tok_rows = self._dispatch_cuda(x, w, ids)
        else:  # CPU tensors (gloo tests): the same plan restated with torch ops
            send_tok, send_counts, send_ids, send_w = plan_dispatch(ids, w, self.E_local, self.world)
            send_x = x.index_select(0, send_tok)
            send_meta = torch.cat([send_ids, send_w.view(torch.int32)], dim=1).contiguous()
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        s_split = send_counts.tolist()
        r_split = recv_counts.tolist()
        S, R = int(sum(s_split)), int(sum(r_split))
        send_x, send_meta = send_x[:S], send_meta[:S]
        recv_x = torch.empty(R, K, dtype=x.dtype, device=x.device)
        recv_meta = torch.empty(R, 2 * self.topk, dtype=torch.int32, device=x.device)
        self._mark("plan")
        dist.all_to_all_single(recv_x, send_x, output_split_sizes=r_split, input_split_sizes=s_split,
                               group=self.group)
        dist.all_to_all_single(recv_meta, send_meta, output_split_sizes=r_split, input_split_sizes=s_split,
                               group=self.group)
        recv_ids = recv_meta[:, : self.topk].contiguous()
        recv_w = recv_meta[:, self.topk:].contiguous().view(torch.float32)
        self._mark("dispatch")
        partial = self.expert_fn(recv_x, recv_w, recv_ids, events=events)
        self._mark("experts")
        back = torch.empty(S, K, dtype=partial.dtype, device=x.device)
        dist.all_to_all_single(back, partial.contiguous(), output_split_sizes=s_split, input_split_sizes=r_split,
                               group=self.group)
        self._mark("combine_a2a")
        if x.is_cuda:
            out = self._combine_cuda(back, tok_rows, M, K, x.dtype)
        else:
            out = torch.zeros(M, K, dtype=torch.float32, device=x.device)
            out.index_add_(0, send_tok, back.float())
            out = out.to(x.dtype)
        self._mark("reduce")
        self._last_recv_ids = recv_ids
        if self.profile and self._marks:
            self.phase_log.append(self._marks)
        return out

    # ------------------------------------------------------------------ CUDA dispatch / combine
    def _dispatch_cuda(self, x, w, ids):
        """Count, scan and pack with the library's EP kernels (one host-visible output: the counts)."""
        from . import _lib
        from .ops import _DTYPES, _ptr, _stream

        M, K = x.shape
        lib = _lib.load()
        cap = max(1, int(lib.moe_ep_send_capacity(M, self.topk, self.world)))
        dev = x.device
        key = (cap, K, x.dtype)
        if getattr(self, "_buf_key", None) != key:
            self._buf_key = key
            self._send_x = torch.empty(cap, K, dtype=x.dtype, device=dev)
            self._send_meta = torch.empty(cap, 2 * self.topk, dtype=torch.int32, device=dev)
            self._scratch = torch.empty(2 * self.world + 1, dtype=torch.int32, device=dev)
            self._offsets = torch.empty(self.world + 1, dtype=torch.int32, device=dev)
            self._counts = torch.empty(self.world, dtype=torch.int64, device=dev)
        tok_rows = torch.empty(M, self.world, dtype=torch.int32, device=dev)
        xc = x.contiguous()
        ids32 = ids.to(torch.int32).contiguous()
        w32 = w.to(torch.float32).contiguous()
        st = _stream(dev)
        _lib.check(lib.moe_ep_plan(_ptr(ids32), M, self.topk, self.E_local, self.world, _ptr(self._scratch),
                                   _ptr(self._offsets), _ptr(self._counts), st), "moe_ep_plan")
        _lib.check(lib.moe_ep_pack(_DTYPES[x.dtype], _ptr(xc), _ptr(ids32), _ptr(w32), M, K, self.topk, self.E_local,
                                   self.world, _ptr(self._scratch), _ptr(self._offsets), _ptr(self._send_x),
                                   _ptr(self._send_meta), _ptr(tok_rows), st), "moe_ep_pack")
        return self._send_x, self._send_meta, self._counts, tok_rows

    def _combine_cuda(self, back, tok_rows, M, K, dtype):
        from . import _lib
        from .ops import _DTYPES, _ptr, _stream

        out = torch.empty(M, K, dtype=dtype, device=back.device)
        if back.numel() == 0:
            back = torch.empty(1, K, dtype=dtype, device=back.device)  # valid pointer; no row is read
        _lib.check(_lib.load().moe_ep_combine(_DTYPES[dtype], _ptr(back), _ptr(tok_rows), M, K, self.world, _ptr(out),
                                              _stream(back.device)), "moe_ep_combine")
        return out

    def phase_breakdown(self):
        """Mean ms per phase over the profiled forwards (synchronises)."""
        torch.cuda.synchronize()
        acc = {}
        for marks in self.phase_log:
            for (n0, e0), (n1, e1) in zip(marks, marks[1:]):
                acc.setdefault(n1, []).append(e0.elapsed_time(e1))
        return {k: sum(v) / len(v) for k, v in acc.items()}

    __call__ = forward

    def local_work(self):
        """(valid local pairs, distinct local experts) of the last forward (synchronises)."""
        ids = self._last_recv_ids
        valid = ids[ids >= 0]
        return int(valid.numel()), int(torch.unique(valid).numel())

    def e2e(self, x, gating, steps: int = 3):
        """tokens/s of the whole job through forward() with host buffers (pinned H2D in, D2H out)."""
        xh = x.cpu().pin_memory()
        gh = gating.cpu().pin_memory()
        oh = torch.empty_like(xh).pin_memory()
        xd, gd = torch.empty_like(x), torch.empty_like(gating)
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            xd.copy_(xh, non_blocking=True)
            gd.copy_(gh, non_blocking=True)
            o = self.forward(xd, gd)
            oh.copy_(o, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        ms = torch.tensor([a.elapsed_time(b) / steps], device=x.device)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX, group=self.group)
        ms = float(ms.item())
        m_total = x.shape[0] * self.world
        return {"value": m_total / (ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": xh.numel() * xh.element_size() + gh.numel() * gh.element_size(),
                "d2h_bytes_per_step": oh.numel() * oh.element_size(), "ms_per_step": ms,
                "note": "per-rank host bytes; value is the whole job"}

    def close(self):
        self._ws = None
