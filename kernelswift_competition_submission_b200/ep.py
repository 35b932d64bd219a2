"""Expert-parallel MoE layer (one process per GPU; NCCL all-to-all or NVLink peer stores).

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

``transport="p2p"`` replaces steps 3 and 5 by NVLink stores into per-rank arenas
shared through CUDA IPC (``moe_p2p_*``): no NCCL call and no host read of split
sizes inside a step, and the expert combine is fused with the return stores.

FP8 w8a8 (``use_fp8_w8a8=True``, e4m3 expert weights with fp32 scales per
128 x 128 block): each rank quantises its own token rows once, per token per
128 (``quant_fn``, default ``quantize_rows_fp8_packed``), and the dispatch moves
the packed e4m3 rows (K codes + K / 128 fp32 scales: 7392 bytes at K = 7168
instead of 14336 in bf16); the receiving rank runs the FP8 expert path straight
from those rows and returns bf16 partial rows. The quantisation is per token, so
every pair sees the same operands as in the single-GPU FP8 path.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist


def _lib_load():
    from . import _lib

    return _lib.load()


def plan_dispatch(ids: torch.Tensor, w: torch.Tensor, experts_per_rank: int, world: int,
                  expert_map: torch.Tensor | None = None):
    """Deduplicated per-destination send list for routed tokens.

    ids int [M, k] global expert ids, w float [M, k]. Expert e lives on rank
    e // experts_per_rank as local expert e % experts_per_rank, or, with
    ``expert_map`` (int [E], (rank << 16) | local id), where the map puts it.
    Returns (send_tok int64 [S], send_counts int64 [world], send_ids int32 [S, k], send_w fp32 [S, k]),
    rows ordered by destination rank then token.
    """
    M, k = ids.shape
    ids64 = ids.long()
    n_exp = experts_per_rank * world if expert_map is None else expert_map.numel()
    valid = (ids64 >= 0) & (ids64 < n_exp)
    if expert_map is None:
        dst = torch.div(ids64, experts_per_rank, rounding_mode="floor").clamp(0, world - 1)
        loc = ids64 - dst * experts_per_rank
    else:
        m = expert_map.long()[ids64.clamp(0, n_exp - 1)]
        dst = (m >> 16).clamp(0, world - 1)
        loc = m & 0xFFFF
    hit = torch.zeros(M, world, dtype=torch.int32, device=ids.device)
    hit.scatter_add_(1, dst, valid.to(torch.int32))
    hit = hit > 0
    send_dst, send_tok = hit.t().nonzero(as_tuple=True)  # sorted by destination, then token
    send_counts = hit.sum(0).to(torch.int64)
    own = (dst[send_tok] == send_dst[:, None]) & valid[send_tok]
    local = loc[send_tok]
    send_ids = torch.where(own, local, torch.full_like(local, -1)).to(torch.int32)
    send_w = w[send_tok].to(torch.float32)
    return send_tok, send_counts, send_ids, send_w


class ExpertParallelMoE:
    """MoE layer with experts sharded over the ranks of ``group``.

    w1_local [E/G, 2N, K], w2_local [E/G, K, N]: this rank's experts.
    """

    def __init__(self, w1_local, w2_local, *, num_experts, topk, num_expert_group=1, topk_group=1,
                 scoring_func="softmax", routed_scaling_factor=1.0, e_score_correction_bias=None,
                 renormalize=True, group=None, route_fn=None, expert_fn=None, chunks=None, reserve_sms=8,
                 transport="nccl", max_tokens=None, use_fp8_w8a8=False, w1_scale=None, w2_scale=None,
                 quant_fn=None, p2p_fused_return=None, p2p_chunk_tokens=512):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"num_experts {num_experts} must divide by the world size {self.world}")
        self.E = num_experts
        self.E_local = num_experts // self.world
        if w1_local.shape[0] != self.E_local or w2_local.shape[0] != self.E_local:
            raise ValueError("w1_local / w2_local must hold num_experts / world experts")
        self.fp8 = bool(use_fp8_w8a8)
        self.w1s = self.w2s = None
        self.scale_format = None
        if self.fp8:
            from .ops import _fp8_bytes, weights_scale_format

            if w1_scale is None or w2_scale is None:
                raise ValueError("use_fp8_w8a8 needs w1_scale and w2_scale")
            El, twoN, Kh = w1_local.shape
            if tuple(w2_local.shape) != (El, Kh, twoN // 2) or Kh % 128 or twoN % 256:
                raise ValueError("use_fp8_w8a8: w1_local [E/G, 2N, K] and w2_local [E/G, K, N], K and N % 128 == 0")
            if tuple(w1_scale.shape) != (El, twoN // 128, Kh // 128) or \
                    tuple(w2_scale.shape) != (El, Kh // 128, twoN // 2 // 128):
                raise ValueError("use_fp8_w8a8: w1_scale / w2_scale must be [E/G, 2N/128, K/128] / [E/G, K/128, N/128]")
            w1_local, w2_local = _fp8_bytes(w1_local.contiguous()), _fp8_bytes(w2_local.contiguous())
            self.w1s = w1_scale.to(torch.float32).contiguous()
            self.w2s = w2_scale.to(torch.float32).contiguous()
            # power-of-two weight scales: the token rows are quantised with power-of-two scales too
            self.scale_format = weights_scale_format(self.w1s, self.w2s)
        self.w1, self.w2 = w1_local, w2_local
        self.hidden = w2_local.shape[1]
        self.quant_fn = quant_fn or self._quant_cuda
        self.topk = topk
        self.route_kw = dict(topk=topk, renormalize=renormalize, num_expert_group=num_expert_group,
                             topk_group=topk_group, scoring_func=scoring_func,
                             routed_scaling_factor=routed_scaling_factor,
                             e_score_correction_bias=e_score_correction_bias)
        self.route_fn = route_fn or self._route_cuda
        self.expert_fn = expert_fn or self._experts_cuda
        self._ws = None
        # per-phase CUDA events of each forward when `profile` is set (bench breakdown)
        self.profile = False
        self.phase_log = []
        self._on_cuda = False
        self._marks = []
        # overlap (chunks > 1): the rank's tokens go in `chunks` pieces; all-to-alls run on a
        # side stream and the expert GEMMs leave `reserve_sms` SMs free for them. Default: 2
        # chunks from 4 ranks up, none below. Measured on B200 (DeepSeek-V3 layer, 32768 tokens):
        # 8 GPUs 6.88 M tokens/s without, 7.16 M with 2 chunks / 16 SMs, 7.69 M with 2 chunks /
        # 8 SMs; 2 GPUs 2.57 M without, 2.27 M with 2 chunks / 16 SMs (all-to-alls small there).
        # With transport="p2p", chunks > 1 is opt-in: measured on 2 GPUs (32768 tokens) the chunked
        # peer-memory layer took 13.1-13.8 ms against 11.1 ms in one piece (each chunk re-reads
        # every local expert's weights and halves the rows per expert).
        if chunks is None:
            chunks = 2 if self.world >= 4 and transport == "nccl" else 1
        self.chunks = max(1, int(chunks))
        self.reserve_sms = max(0, int(reserve_sms))
        self._comm = None
        self._bufs = {}
        self.gemm_log = []  # (gemm1 ms, gemm2 ms, local pairs) per chunk, when profiling
        self._expert_map = None  # int32 [E]: (rank << 16) | local id, set by replicate()
        self.replicated = []
        # transport "p2p": dispatch / combine by NVLink stores into the other ranks' arenas
        # (CUDA IPC), no NCCL and no host round trip per step; for decode-sized batches
        if transport not in ("nccl", "p2p"):
            raise ValueError(f"transport must be 'nccl' or 'p2p', not {transport!r}")
        self.transport = transport
        self.max_tokens = max_tokens  # p2p arena size in tokens per rank (default: the first batch, max over ranks)
        # bf16 p2p return: True = the down GEMM's epilogue stores each finished row into its
        # source's arena; False = scatter GEMM, then a combine-and-return kernel (same bits);
        # None = the fused return up to 4096 received rows per rank (world * max_tokens), where
        # it hides the return under the GEMM, the separate kernels above it, where a row's last
        # slot lands late in the GEMM and the returns would bunch up at its end. The choice
        # depends only on the arena size, so every rank makes the same one.
        self.p2p_fused_return = p2p_fused_return
        # p2p with chunks > 1: one arena per chunk when every chunk holds at least this many
        # tokens per rank (prefill); smaller batches keep one arena (decode)
        self.p2p_chunk_tokens = max(1, int(p2p_chunk_tokens))
        self._p2p = None
        self._p2p_cap = 0
        self._last_recv_ids = None
        self._ws_chunks = []  # expert-path workspaces of the chunked peer-memory forward
        # p2p failure detection: each forward ends with an asynchronous copy of the device
        # status word to pinned host memory; a later forward reads it once that copy is done
        self._p2p_status = None      # (pinned host int32 [1], event) of the last forward
        self._p2p_failed = 0         # failure code seen; sticky until reset_transport()

    @property
    def kernel_launches_per_step(self):
        """This library's kernels launched by one CUDA forward."""
        if self.transport == "p2p":
            # routing, then per arena (one, or one per token chunk): signal, dispatch, wait, align
            # count, align scatter, GEMM1, then bf16: set-up of the fused return + GEMM2 with the
            # combine and return in its epilogue, or GEMM2 + the combine-and-return kernel; FP8:
            # GEMM2 + fused combine-and-return (+ row gather, scale gather, and the quantiser
            # once per step); then wait, reduce
            n = len(self._p2p) if self._p2p else 1
            return 2 + 12 * n if self.fp8 else 1 + 10 * n
        # routing, then per chunk: EP count, EP pack, align count, align scatter, GEMM1, GEMM2,
        # combine, EP combine (FP8: + quantise once, row and scale gathers per chunk)
        return (2 + 10 * self.chunks) if self.fp8 else (1 + 8 * self.chunks)

    # ------------------------------------------------------------------ hot-expert replicas
    def replicate(self, expert_ids, w1_rep, w2_rep, w1s_rep=None, w2s_rep=None):
        """Keep replicas of ``expert_ids`` (weights w1_rep [R, 2N, K], w2_rep [R, K, N], the
        same on every rank; with FP8 weights also their block scales w1s_rep, w2s_rep) on this
        rank and compute their pairs where the token lives.

        Every rank must call it with the same ids. Pairs routed to a replicated expert then
        never cross the network and spread over all ranks with the tokens, instead of all
        landing on the expert's owner; the other experts keep their owner. The result is the
        same layer: each pair is still computed once, with the same weights.
        """
        ids = [int(e) for e in expert_ids]
        if len(set(ids)) != len(ids) or any(e < 0 or e >= self.E for e in ids):
            raise ValueError("replicate: expert ids must be distinct and in [0, num_experts)")
        if w1_rep.shape[0] != len(ids) or w2_rep.shape[0] != len(ids):
            raise ValueError("replicate: one weight slice per replicated expert")
        if self.E_local + len(ids) > 0xFFFF:
            raise ValueError("replicate: too many local experts")
        base_w1 = self.w1[: self.E_local]
        base_w2 = self.w2[: self.E_local]
        if self.fp8:
            from .ops import _fp8_bytes

            if w1s_rep is None or w2s_rep is None or w1s_rep.shape[0] != len(ids) or w2s_rep.shape[0] != len(ids):
                raise ValueError("replicate: FP8 weights need one scale block per replicated expert")
            w1_rep, w2_rep = _fp8_bytes(w1_rep), _fp8_bytes(w2_rep)
            b1s, b2s = self.w1s[: self.E_local], self.w2s[: self.E_local]
            self.w1s = torch.cat([b1s, w1s_rep.to(torch.float32)], dim=0).contiguous() if ids else b1s
            self.w2s = torch.cat([b2s, w2s_rep.to(torch.float32)], dim=0).contiguous() if ids else b2s
        self.w1 = torch.cat([base_w1, w1_rep.to(base_w1.dtype)], dim=0).contiguous() if ids else base_w1
        self.w2 = torch.cat([base_w2, w2_rep.to(base_w2.dtype)], dim=0).contiguous() if ids else base_w2
        emap = [((e // self.E_local) << 16) | (e % self.E_local) for e in range(self.E)]
        for j, e in enumerate(ids):
            emap[e] = (self.rank << 16) | (self.E_local + j)
        self.replicated = ids
        self._expert_map = torch.tensor(emap, dtype=torch.int32, device=self.w1.device) if ids else None

    def rebalance(self, topk_ids, n):
        """Replicate the n busiest experts of ``topk_ids`` (summed over ranks) on every rank,
        their weights broadcast from their owners (collective: every rank calls it with its
        own routing sample). Returns the replicated expert ids."""
        hot = self.hot_experts(topk_ids, n)
        base = [self.w1[: self.E_local], self.w2[: self.E_local]]
        if self.fp8:
            base += [self.w1s[: self.E_local], self.w2s[: self.E_local]]
        reps = [torch.empty((len(hot),) + tuple(b.shape[1:]), dtype=b.dtype, device=b.device) for b in base]
        for j, e in enumerate(hot):
            owner = e // self.E_local
            src = dist.get_global_rank(self.group, owner) if self.group is not None else owner
            for b, r in zip(base, reps):
                if owner == self.rank:
                    r[j].copy_(b[e % self.E_local])
                dist.broadcast(r[j], src=src, group=self.group)
        self.replicate(hot, *reps)
        return hot

    def hot_experts(self, topk_ids, n):
        """The n experts with the most (token, slot) pairs in ``topk_ids`` summed over all
        ranks (ties to the lower id): the candidates for ``replicate``."""
        cnt = torch.bincount(topk_ids.reshape(-1).long().clamp(0, self.E - 1), minlength=self.E).to(torch.int64)
        if dist.get_backend(self.group) == "nccl" and not cnt.is_cuda:
            cnt = cnt.cuda()
        dist.all_reduce(cnt, group=self.group)
        order = sorted(range(self.E), key=lambda e: (-int(cnt[e]), e))
        return order[:n]

    # ------------------------------------------------------------------ default (CUDA) stages
    def _route_cuda(self, x, gating):
        from .ops import grouped_topk

        kw = self.route_kw
        return grouped_topk(x, gating, kw["topk"], kw["renormalize"], kw["num_expert_group"], kw["topk_group"],
                            kw["scoring_func"], kw["routed_scaling_factor"], kw["e_score_correction_bias"])

    def _quant_cuda(self, x):
        from .ops import quantize_rows_fp8_packed

        return quantize_rows_fp8_packed(x, scale_format=self.scale_format)

    def _experts_cuda(self, x, w, ids, events=None, out=None, max_ctas=0):
        from .ops import fused_moe_staged, fused_moe_workspace_bytes

        M = x.shape[0]
        if M == 0:
            if events:
                for e in events:
                    e.record()
            if out is not None:
                return out
            return torch.empty(0, self.hidden, dtype=torch.bfloat16 if self.fp8 else x.dtype, device=x.device)
        if self.fp8:  # x: packed e4m3 rows
            from .ops import fused_moe_fp8_rows

            need = int(_lib_load().moe_fused_workspace_bytes_fp8(M, self.w1.shape[0], ids.shape[1], self.hidden,
                                                                 self.w2.shape[2]))
            if self._ws is None or self._ws.numel() < need:
                self._ws = torch.empty(int(need * 1.25) + 256, dtype=torch.uint8, device=x.device)
            if events:  # one library call: the stage events bracket it (no per-GEMM split)
                events[0].record()
            y = fused_moe_fp8_rows(x, self.hidden, self.w1, self.w1s, self.w2, self.w2s, w, ids, out=out,
                                   workspace=self._ws, max_ctas=max_ctas, scale_format=self.scale_format)
            if events:
                for e in events[1:]:
                    e.record()
            return y
        need = fused_moe_workspace_bytes(M, self.w1.shape[0], ids.shape[1], x.shape[1], self.w2.shape[2])
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(int(need * 1.25) + 256, dtype=torch.uint8, device=x.device)
        return fused_moe_staged(x, self.w1, self.w2, w, ids, workspace=self._ws, events=events, out=out,
                                max_ctas=max_ctas)

    def _buf(self, name, rows, cols, dtype, dev):
        """Persistent, grow-only buffer: a tensor handed to another stream is never freed mid-step."""
        t = self._bufs.get(name)
        if t is None or t.shape[0] < rows or t.shape[1] != cols or t.dtype != dtype:
            t = torch.empty(max(1, int(rows * 1.2) + 16), cols, dtype=dtype, device=dev)
            self._bufs[name] = t
        return t

    # ------------------------------------------------------------------ forward
    def _mark(self, name):
        if self.profile and self._on_cuda:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._marks.append((name, ev))

    def forward(self, x: torch.Tensor, gating: torch.Tensor, events=None) -> torch.Tensor:
        if self.fp8 and x.is_cuda and x.dtype != torch.bfloat16:
            raise TypeError("use_fp8_w8a8: hidden states must be bf16")
        if x.is_cuda and self.transport == "p2p":
            return self._forward_p2p(x, gating)
        if x.is_cuda and self.chunks > 1 and self.expert_fn == self._experts_cuda:
            return self._forward_overlapped(x, gating, events)
        return self._forward_simple(x, gating, events)

    def _forward_simple(self, x: torch.Tensor, gating: torch.Tensor, events=None) -> torch.Tensor:
        M, K = x.shape
        self._on_cuda = x.is_cuda
        self._marks = []
        self._mark("start")
        w, ids = self.route_fn(x, gating)
        self._mark("route")
        payload = self.quant_fn(x) if self.fp8 else x  # the rows that travel
        if x.is_cuda:
            send_x, send_meta, send_counts, tok_rows = self._dispatch_cuda(payload, w, ids, hidden=K)
        else:  # CPU tensors (gloo tests): the same plan restated with torch ops
            send_tok, send_counts, send_ids, send_w = plan_dispatch(ids, w, self.E_local, self.world,
                                                                    self._expert_map)
            send_x = payload.index_select(0, send_tok)
            send_meta = torch.cat([send_ids, send_w.view(torch.int32)], dim=1).contiguous()
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        s_split = send_counts.tolist()
        r_split = recv_counts.tolist()
        S, R = int(sum(s_split)), int(sum(r_split))
        send_x, send_meta = send_x[:S], send_meta[:S]
        recv_x = torch.empty(R, payload.shape[1], dtype=payload.dtype, device=x.device)
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

    def _forward_overlapped(self, x: torch.Tensor, gating: torch.Tensor, events=None) -> torch.Tensor:
        """Chunked forward: dispatch of chunk c+1 and combine of chunk c run on a side
        stream while the experts of chunk c (then c+1) run on the current stream."""
        from . import _lib
        from .ops import _DTYPES, _ptr, _stream

        M, K = x.shape
        dev = x.device
        C = self.chunks
        cur = torch.cuda.current_stream(dev)
        if self._comm is None:
            self._comm = torch.cuda.Stream(device=dev)
        comm = self._comm
        self._on_cuda = True
        self._marks = []
        self._mark("start")
        w, ids = self.route_fn(x, gating)
        self._mark("route")
        payload = self.quant_fn(x) if self.fp8 else x
        P = payload.shape[1]
        bounds = [(M * c) // C for c in range(C + 1)]
        packs = []
        for c in range(C):
            t0, t1 = bounds[c], bounds[c + 1]
            packs.append(self._dispatch_cuda(payload[t0:t1], w[t0:t1], ids[t0:t1], tag=c, hidden=K))
        # per-chunk row counts, one exchange: send[d, c] rows of chunk c go to rank d
        send_counts = torch.stack([p[2] for p in packs], dim=1).contiguous()  # [world, C] int64
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc = send_counts.tolist()
        rc = recv_counts.tolist()
        s_split = [[sc[d][c] for d in range(self.world)] for c in range(C)]
        r_split = [[rc[d][c] for d in range(self.world)] for c in range(C)]
        self._mark("plan")
        max_ctas = 0
        if self.reserve_sms:
            max_ctas = max(1, torch.cuda.get_device_properties(dev).multi_processor_count - self.reserve_sms)
        ready = torch.cuda.Event()
        ready.record(cur)
        recvs, disp_ev = [], []
        with torch.cuda.stream(comm):
            comm.wait_event(ready)
            for c in range(C):
                S, R = sum(s_split[c]), sum(r_split[c])
                send_x, send_meta = packs[c][0], packs[c][1]
                rx = self._buf(f"rx{c}", R, P, payload.dtype, dev)[:R]
                rm = self._buf(f"rm{c}", R, 2 * self.topk, torch.int32, dev)[:R]
                dist.all_to_all_single(rx, send_x[:S], output_split_sizes=r_split[c], input_split_sizes=s_split[c],
                                       group=self.group)
                dist.all_to_all_single(rm, send_meta[:S], output_split_sizes=r_split[c],
                                       input_split_sizes=s_split[c], group=self.group)
                ev = torch.cuda.Event()
                ev.record(comm)
                recvs.append((rx, rm))
                disp_ev.append(ev)
        self._mark("dispatch_issued")
        partials, exp_ev = [], []
        self.gemm_log_step = []
        for c in range(C):
            cur.wait_event(disp_ev[c])
            rx, rm = recvs[c]
            R = rx.shape[0]
            rids = rm[:, : self.topk].contiguous()
            rw = rm[:, self.topk:].contiguous().view(torch.float32)
            part = self._buf(f"part{c}", R, K, x.dtype, dev)[:R]
            # GEMM-level events: the bf16 stages only (the FP8 path is one library call)
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(5)] if self.profile and not self.fp8 else None
            self._experts_cuda(rx, rw, rids, events=evs, out=part, max_ctas=max_ctas)
            if evs:
                self.gemm_log_step.append((evs, rids))
            ev = torch.cuda.Event()
            ev.record(cur)
            partials.append(part)
            exp_ev.append(ev)
        self._mark("experts")
        backs, back_ev = [], []
        with torch.cuda.stream(comm):
            for c in range(C):
                comm.wait_event(exp_ev[c])
                S = sum(s_split[c])
                back = self._buf(f"back{c}", S, K, x.dtype, dev)[:S]
                dist.all_to_all_single(back, partials[c], output_split_sizes=s_split[c],
                                       input_split_sizes=r_split[c], group=self.group)
                ev = torch.cuda.Event()
                ev.record(comm)
                backs.append(back)
                back_ev.append(ev)
        out = torch.empty(M, K, dtype=x.dtype, device=dev)
        lib = _lib.load()
        for c in range(C):
            cur.wait_event(back_ev[c])
            t0, t1 = bounds[c], bounds[c + 1]
            if t1 > t0:
                back = backs[c] if backs[c].numel() else torch.empty(1, K, dtype=x.dtype, device=dev)
                _lib.check(lib.moe_ep_combine(_DTYPES[x.dtype], _ptr(back), _ptr(packs[c][3]), t1 - t0, K, self.world,
                                              _ptr(out[t0:t1]), _stream(dev)), "moe_ep_combine")
        self._mark("combine")
        self._last_recv_ids = torch.cat([r[1][:, : self.topk] for r in recvs]) if recvs else None
        if self.profile and self._marks:
            self.phase_log.append(self._marks)
            self.gemm_log.append(self.gemm_log_step)
        return out

    # ------------------------------------------------------------------ CUDA dispatch / combine
    def _dispatch_cuda(self, x, w, ids, tag=0, hidden=None):
        """Count, scan and pack with the library's EP kernels (one host-visible output: the counts).
        x: bf16 / fp16 token rows, or packed e4m3 rows (uint8) of a ``hidden``-wide token."""
        from . import _lib
        from .ops import _DTYPES, _ptr, _stream

        M, C = x.shape
        K = hidden or C
        dt = _lib.MOE_DTYPE_E4M3_ROW if x.dtype == torch.uint8 else _DTYPES[x.dtype]
        lib = _lib.load()
        cap = max(1, int(lib.moe_ep_send_capacity(M, self.topk, self.world)))
        dev = x.device
        send_x = self._buf(f"sx{tag}", cap, C, x.dtype, dev)
        send_meta = self._buf(f"sm{tag}", cap, 2 * self.topk, torch.int32, dev)
        scratch = self._buf(f"scr{tag}", 2 * self.world + 1, 1, torch.int32, dev)
        offsets = self._buf(f"off{tag}", self.world + 1, 1, torch.int32, dev)
        counts = torch.empty(self.world, dtype=torch.int64, device=dev)
        tok_rows = self._buf(f"tr{tag}", max(M, 1), self.world, torch.int32, dev)[: max(M, 1)]
        xc = x.contiguous()
        ids32 = ids.to(torch.int32).contiguous()
        w32 = w.to(torch.float32).contiguous()
        st = _stream(dev)
        if self._expert_map is None:
            _lib.check(lib.moe_ep_plan(_ptr(ids32), M, self.topk, self.E_local, self.world, _ptr(scratch),
                                       _ptr(offsets), _ptr(counts), st), "moe_ep_plan")
            _lib.check(lib.moe_ep_pack(dt, _ptr(xc), _ptr(ids32), _ptr(w32), M, K, self.topk,
                                       self.E_local, self.world, _ptr(scratch), _ptr(offsets), _ptr(send_x),
                                       _ptr(send_meta), _ptr(tok_rows), st), "moe_ep_pack")
        else:
            emap = self._expert_map
            if emap.device != dev:
                emap = self._expert_map = emap.to(dev)
            _lib.check(lib.moe_ep_plan_mapped(_ptr(ids32), M, self.topk, self.E, _ptr(emap), self.world,
                                              _ptr(scratch), _ptr(offsets), _ptr(counts), st), "moe_ep_plan_mapped")
            _lib.check(lib.moe_ep_pack_mapped(dt, _ptr(xc), _ptr(ids32), _ptr(w32), M, K, self.topk,
                                              self.E, _ptr(emap), self.world, _ptr(scratch), _ptr(offsets),
                                              _ptr(send_x), _ptr(send_meta), _ptr(tok_rows), st),
                       "moe_ep_pack_mapped")
        return send_x, send_meta, counts, tok_rows

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

    def gemm_breakdown(self):
        """Mean over profiled forwards of (GEMM1 ms, GEMM2 ms, valid local pairs), summed over chunks."""
        torch.cuda.synchronize()
        tot = []
        for step in self.gemm_log:
            g1 = sum(e[1].elapsed_time(e[2]) for e, _ in step)
            g2 = sum(e[2].elapsed_time(e[3]) for e, _ in step)
            pairs = sum(int((r >= 0).sum()) for _, r in step)
            tot.append((g1, g2, pairs))
        if not tot:
            return None
        n = len(tot)
        return tuple(sum(t[i] for t in tot) / n for i in range(3))

    def local_work(self):
        """(valid local pairs, distinct local experts) of the last forward (synchronises)."""
        ids = self._last_recv_ids
        if ids is None:
            return 0, 0
        valid = ids[ids >= 0]
        return int(valid.numel()), int(torch.unique(valid).numel())

    # ------------------------------------------------------------------ NVLink peer-memory transport
    def _p2p_setup(self, M, K, dtype, dev):
        """Collective: the arenas of this layer for `cap` tokens per rank (the largest local
        batch over the ranks): one arena, or with chunks > 1 one per chunk of ceil(cap / chunks)
        tokens, each with its own flags and sequence numbers."""
        self._p2p_release()
        m = torch.tensor([M], dtype=torch.int64, device=dev)
        dist.all_reduce(m, op=dist.ReduceOp.MAX, group=self.group)
        cap = max(1, int(m.item()))
        C = self.chunks if cap // max(1, self.chunks) >= self.p2p_chunk_tokens else 1
        self._p2p_cap = cap
        capc = cap if C == 1 else -(-cap // C)
        self._p2p = [self._p2p_arena(capc, K, dtype, dev) for _ in range(C)]
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    def _p2p_arena(self, cap, K, dtype, dev):
        """Collective: allocate this rank's arena for `cap` tokens per source rank, exchange
        the CUDA IPC handles and open the other ranks' arenas."""
        from . import _lib

        lib = _lib.load()
        nbytes = int(lib.moe_p2p_arena_bytes(self.world, cap, K, self.topk))
        if nbytes <= 0:
            raise ValueError("p2p transport: unsupported shape")
        base = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        _lib.check(lib.moe_p2p_alloc(self.world, cap, K, self.topk, ctypes.cast(ctypes.pointer(base), ctypes.c_void_p),
                                     handle), "moe_p2p_alloc")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=self.group)
        bases = []
        for r, h in enumerate(handles):
            if r == self.rank:
                bases.append(base.value)
            else:
                pb = ctypes.c_void_p()
                _lib.check(lib.moe_p2p_open(ctypes.create_string_buffer(h, 64),
                                            ctypes.cast(ctypes.pointer(pb), ctypes.c_void_p)), "moe_p2p_open")
                bases.append(pb.value)
        offs = (ctypes.c_int64 * 9)()
        _lib.check(lib.moe_p2p_arena_offsets(self.world, cap, K, self.topk, offs), "moe_p2p_arena_offsets")
        return {
            "cap": cap, "K": K, "dtype": dtype, "base": base.value, "bases": bases, "offs": list(offs), "seq": 0,
            "peer_bases": torch.tensor(bases, dtype=torch.int64, device=dev),
            "scr_d": torch.zeros(2 * self.world + 1, dtype=torch.int32, device=dev),
            "scr_c": torch.zeros(max(1, self.world), dtype=torch.int32, device=dev),
        }

    def _p2p_release(self):
        if self._p2p is None:
            return
        from . import _lib

        lib = _lib.load()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no rank still writes into an arena being unmapped
        for a in self._p2p:
            for r, b in enumerate(a["bases"]):
                if r != self.rank:
                    lib.moe_p2p_close(ctypes.c_void_p(b))
        dist.barrier(group=self.group)
        for a in self._p2p:
            lib.moe_p2p_free(ctypes.c_void_p(a["base"]))
        self._p2p = None

    # ------------------------------------------------------------------ p2p failure handling
    def _p2p_raise_if_failed(self, block=False):
        """Raise once a peer-memory step of this rank recorded a device-side failure (a wait
        that gave up after its 2 s limit). Reads the host copy of the status word that the
        last forward queued; with ``block`` it waits for that copy, otherwise a copy still in
        flight is left for a later call. The failure is sticky until ``reset_transport()``."""
        if not self._p2p_failed and self._p2p_status is not None:
            host, ev = self._p2p_status
            if block:
                ev.synchronize()
            if ev.query() and int(host[0]):
                self._p2p_failed = int(host[0])
        if self._p2p_failed:
            from . import _lib

            raise RuntimeError(
                f"expert-parallel peer-memory transport failed on rank {self.rank}: "
                f"{_lib.status_string(self._p2p_failed)}; the steps since then returned NaN rows. "
                "Call reset_transport() on every rank to rebuild the arenas.")

    def check_transport(self):
        """Synchronise with this rank's last peer-memory step and raise if it failed."""
        self._p2p_raise_if_failed(block=True)

    def reset_transport(self):
        """Collective (every rank): after a peer-memory failure, zero the status word, unmap
        and free the arenas; the next forward allocates and exchanges new ones."""
        from .ops import status_word

        if self._p2p is None and not self._p2p_failed:
            return
        torch.cuda.synchronize()
        dev = torch.device("cuda", torch.cuda.current_device())
        status_word(dev).zero_()
        self._p2p_failed = 0
        self._p2p_status = None
        self._p2p_release()

    def _forward_p2p(self, x, gating):
        from . import _lib
        from .ops import _DTYPES, _ptr, _stream, status_word

        self._p2p_raise_if_failed()
        M, K = x.shape
        dev = x.device
        if self._p2p is None:  # collective: the first forward of every rank
            self._p2p_setup(max(M, int(self.max_tokens or 0)), K, x.dtype, dev)
        p = self._p2p[0]
        if M > self._p2p_cap or K != p["K"] or x.dtype != p["dtype"]:
            raise ValueError(f"p2p transport: batch [{M}, {K}] {x.dtype} does not fit the arena "
                             f"(max_tokens {self._p2p_cap}, hidden {p['K']}, {p['dtype']})")
        if len(self._p2p) > 1:
            return self._forward_p2p_chunked(x, gating)
        lib = _lib.load()
        st = _stream(dev)
        status = _ptr(status_word(dev))
        dt = _DTYPES[x.dtype]
        W, cap, k = self.world, p["cap"], self.topk
        p["seq"] = (p["seq"] + 1) & 0xFFFFFFFF or 1
        seq = p["seq"]
        self._on_cuda = True
        self._marks = []
        self._mark("start")
        w, ids = self.route_fn(x, gating)
        self._mark("route")
        # the rows that travel: the token rows, or their packed e4m3 form (FP8)
        xc = self.quant_fn(x) if self.fp8 else x.contiguous()
        dt_rows = _lib.MOE_DTYPE_E4M3_ROW if self.fp8 else dt
        ids32 = ids.to(torch.int32).contiguous()
        w32 = w.to(torch.float32).contiguous()
        tok_rows = self._buf("p2p_tr", max(M, 1), W, torch.int32, dev)[: max(M, 1)]
        pb = _ptr(p["peer_bases"])
        base = p["base"]
        _lib.check(lib.moe_p2p_signal(pb, W, self.rank, 0, cap, K, k, seq, status, st), "moe_p2p_signal")
        _lib.check(lib.moe_p2p_dispatch(dt_rows, _ptr(xc), _ptr(ids32), _ptr(w32), M, K, k, self.E_local, W, self.rank,
                                        cap, pb, base, seq, _ptr(p["scr_d"]), _ptr(tok_rows), status, st),
                   "moe_p2p_dispatch")
        _lib.check(lib.moe_p2p_wait(base, W, 1, cap, K, k, seq, status, st), "moe_p2p_wait")
        self._mark("dispatch")
        if self.profile:  # received ids, for local_work() statistics
            rids = torch.empty(W * cap, k, dtype=torch.int32, device=dev)
            _lib.check(lib.moe_p2p_copy_recv_ids(base, W, cap, K, k, _ptr(rids), st), "moe_p2p_copy_recv_ids")
            self._last_recv_ids = rids
        # local experts over every received row (unused rows carry id -1)
        R = W * cap
        o = p["offs"]
        E_l, N = self.w1.shape[0], self.w2.shape[2]
        need = int(lib.moe_fused_workspace_bytes_fp8(R, E_l, k, K, N) if self.fp8 else
                   lib.moe_fused_workspace_bytes(R, E_l, k, K, N))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(int(need * 1.25) + 256, dtype=torch.uint8, device=dev)
        ws, wsn = _ptr(self._ws), self._ws.numel()
        rx, rid = base + o[4], base + o[5]
        if self.fp8:  # GEMMs straight from the received packed rows; the slot rows stay in ws
            _lib.check(lib.moe_fused_experts_fp8_rows(ctypes.c_void_p(rx), int(lib.moe_fp8_row_bytes(K)),
                                                      _ptr(self.w1), _ptr(self.w1s), _ptr(self.w2), _ptr(self.w2s),
                                                      None, ctypes.c_void_p(rid), R, E_l, k, K, N,
                                                      _lib.MOE_FP8_SCALE_UE8M0 if self.scale_format == "ue8m0"
                                                      else _lib.MOE_FP8_SCALE_FP32, None, ws, wsn, 0, status, st),
                                   "moe_fused_experts_fp8_rows")
            self._mark("experts")
            # top-k combine of each valid received row, stored straight into its source's arena
            _lib.check(lib.moe_p2p_combine_experts_back(dt_rows, ws, E_l, K, N, k, W, self.rank, cap, pb, base, seq,
                                                        _ptr(p["scr_c"]), status, st), "moe_p2p_combine_experts_back")
        else:
            _lib.check(lib.moe_expert_align_gather(dt, ctypes.c_void_p(rx), ctypes.c_void_p(rid), R, E_l, k, K, N,
                                                   ws, wsn, st), "moe_expert_align_gather")
            _lib.check(lib.moe_expert_gemm1(dt, _ptr(self.w1), R, E_l, k, K, N, ws, wsn, status, 0, st),
                       "moe_expert_gemm1")
            fused = self.p2p_fused_return if self.p2p_fused_return is not None else R <= 4096
            if fused:
                # the down GEMM's epilogue sums each received row's slots and stores the sum into
                # its source rank's arena over NVLink while the GEMM still runs (one kernel)
                _lib.check(lib.moe_p2p_expert_gemm2_return(dt, _ptr(self.w2), ws, wsn, E_l, K, N, k, W, self.rank,
                                                           cap, pb, base, seq, _ptr(p["scr_c"]), status, 0, st),
                           "moe_p2p_expert_gemm2_return")
                self._mark("experts")
            else:
                _lib.check(lib.moe_expert_gemm2(dt, _ptr(self.w2), R, E_l, k, K, N, ws, wsn, status, 0, st),
                           "moe_expert_gemm2")
                self._mark("experts")
                _lib.check(lib.moe_p2p_combine_experts_back(dt, ws, E_l, K, N, k, W, self.rank, cap, pb, base, seq,
                                                            _ptr(p["scr_c"]), status, st),
                           "moe_p2p_combine_experts_back")
        _lib.check(lib.moe_p2p_wait(base, W, 2, cap, K, k, seq, status, st), "moe_p2p_wait")
        self._mark("combine_back")
        out = torch.empty(M, K, dtype=x.dtype, device=dev)
        if M:  # NaN rows if any wait of this step gave up
            _lib.check(lib.moe_p2p_reduce(dt, base, _ptr(tok_rows), M, K, k, W, cap, _ptr(out), status, st),
                       "moe_p2p_reduce")
        self._mark("reduce")
        # the status word, copied to the host behind this step (read by a later forward)
        if self._p2p_status is None:
            self._p2p_status = (torch.zeros(1, dtype=torch.int32).pin_memory(), torch.cuda.Event())
        host, ev = self._p2p_status
        host.copy_(status_word(dev), non_blocking=True)
        ev.record()
        if self.profile and self._marks:
            self.phase_log.append(self._marks)
        return out

    def _forward_p2p_chunked(self, x, gating):
        """Peer-memory transport in token chunks, one arena per chunk (own flags, own sequence
        numbers). Chunk 0 is dispatched on the current stream and the others on a side stream,
        under chunk 0's experts; each chunk's combine-and-return runs on the side stream under
        the next chunk's experts; the sums per token come last. The expert GEMMs leave
        `reserve_sms` SMs to the transport kernels. A wait kernel never spins on a flag that a
        kernel of its own GPU has still to write: before it, its stream waits (CUDA event) for
        this rank's own kernel of that phase, so only the other ranks' kernels are awaited."""
        from . import _lib
        from .ops import _DTYPES, _ptr, status_word

        M, K = x.shape
        dev = x.device
        arenas = self._p2p
        C = len(arenas)
        lib = _lib.load()
        main = torch.cuda.current_stream(dev)
        if self._comm is None:
            self._comm = torch.cuda.Stream(device=dev)
        side = self._comm
        status = _ptr(status_word(dev))
        dt = _DTYPES[x.dtype]
        W, k = self.world, self.topk
        E_l, N = self.w1.shape[0], self.w2.shape[2]
        for a in arenas:
            a["seq"] = (a["seq"] + 1) & 0xFFFFFFFF or 1
        self._on_cuda = True
        self._marks = []
        self._mark("start")
        w, ids = self.route_fn(x, gating)
        self._mark("route")
        xc = self.quant_fn(x) if self.fp8 else x.contiguous()
        dt_rows = _lib.MOE_DTYPE_E4M3_ROW if self.fp8 else dt
        ids32 = ids.to(torch.int32).contiguous()
        w32 = w.to(torch.float32).contiguous()
        bounds = [(M * c) // C for c in range(C + 1)]
        max_ctas = 0
        if self.reserve_sms:
            max_ctas = max(1, torch.cuda.get_device_properties(dev).multi_processor_count - self.reserve_sms)
        ev_route = torch.cuda.Event()
        ev_route.record(main)
        tok_rows = [self._buf(f"p2p_tr{c}", max(bounds[c + 1] - bounds[c], 1), W, torch.int32, dev)
                    for c in range(C)]
        ev_disp = []
        for c, a in enumerate(arenas):
            s = main if c == 0 else side
            t0, t1 = bounds[c], bounds[c + 1]
            pb = _ptr(a["peer_bases"])
            with torch.cuda.stream(s):
                if c == 1:
                    side.wait_event(ev_route)
                sp = s.cuda_stream
                _lib.check(lib.moe_p2p_signal(pb, W, self.rank, 0, a["cap"], K, k, a["seq"], status, sp),
                           "moe_p2p_signal")
                _lib.check(lib.moe_p2p_dispatch(dt_rows, _ptr(xc[t0:t1]), _ptr(ids32[t0:t1]), _ptr(w32[t0:t1]),
                                                t1 - t0, K, k, E_l, W, self.rank, a["cap"], pb, a["base"], a["seq"],
                                                _ptr(a["scr_d"]), _ptr(tok_rows[c]), status, sp), "moe_p2p_dispatch")
                ev = torch.cuda.Event()
                ev.record(s)
                ev_disp.append(ev)
        if len(self._ws_chunks) != C:
            self._ws_chunks = [None] * C
        ev_back = []
        st_main, st_side = main.cuda_stream, side.cuda_stream
        for c, a in enumerate(arenas):
            base, cap, o = a["base"], a["cap"], a["offs"]
            pb = _ptr(a["peer_bases"])
            main.wait_event(ev_disp[c])
            _lib.check(lib.moe_p2p_wait(base, W, 1, cap, K, k, a["seq"], status, st_main), "moe_p2p_wait")
            if c == 0:
                self._mark("dispatch")
                recv_ids = []
            if self.profile:  # received ids, for local_work() statistics
                rids = torch.empty(W * cap, k, dtype=torch.int32, device=dev)
                _lib.check(lib.moe_p2p_copy_recv_ids(base, W, cap, K, k, _ptr(rids), st_main),
                           "moe_p2p_copy_recv_ids")
                recv_ids.append(rids)
            R = W * cap
            need = int(lib.moe_fused_workspace_bytes_fp8(R, E_l, k, K, N) if self.fp8 else
                       lib.moe_fused_workspace_bytes(R, E_l, k, K, N))
            if self._ws_chunks[c] is None or self._ws_chunks[c].numel() < need:
                self._ws_chunks[c] = torch.empty(int(need * 1.25) + 256, dtype=torch.uint8, device=dev)
            ws, wsn = _ptr(self._ws_chunks[c]), self._ws_chunks[c].numel()
            rx, rid = base + o[4], base + o[5]
            fused = False
            if self.fp8:
                _lib.check(lib.moe_fused_experts_fp8_rows(ctypes.c_void_p(rx), int(lib.moe_fp8_row_bytes(K)),
                                                          _ptr(self.w1), _ptr(self.w1s), _ptr(self.w2),
                                                          _ptr(self.w2s), None, ctypes.c_void_p(rid), R, E_l, k, K, N,
                                                          _lib.MOE_FP8_SCALE_UE8M0 if self.scale_format == "ue8m0"
                                                          else _lib.MOE_FP8_SCALE_FP32, None, ws, wsn, max_ctas,
                                                          status, st_main), "moe_fused_experts_fp8_rows")
            else:
                _lib.check(lib.moe_expert_align_gather(dt, ctypes.c_void_p(rx), ctypes.c_void_p(rid), R, E_l, k, K,
                                                       N, ws, wsn, st_main), "moe_expert_align_gather")
                _lib.check(lib.moe_expert_gemm1(dt, _ptr(self.w1), R, E_l, k, K, N, ws, wsn, status, max_ctas,
                                                st_main), "moe_expert_gemm1")
                fused = self.p2p_fused_return if self.p2p_fused_return is not None else R <= 4096
                if fused:
                    _lib.check(lib.moe_p2p_expert_gemm2_return(dt, _ptr(self.w2), ws, wsn, E_l, K, N, k, W,
                                                               self.rank, cap, pb, base, a["seq"], _ptr(a["scr_c"]),
                                                               status, max_ctas, st_main),
                               "moe_p2p_expert_gemm2_return")
                else:
                    _lib.check(lib.moe_expert_gemm2(dt, _ptr(self.w2), R, E_l, k, K, N, ws, wsn, status, max_ctas,
                                                    st_main), "moe_expert_gemm2")
            ev = torch.cuda.Event()
            ev.record(main)
            if not fused:  # the return of chunk c under the experts of chunk c + 1
                with torch.cuda.stream(side):
                    side.wait_event(ev)
                    _lib.check(lib.moe_p2p_combine_experts_back(dt_rows, ws, E_l, K, N, k, W, self.rank, cap, pb,
                                                                base, a["seq"], _ptr(a["scr_c"]), status, st_side),
                               "moe_p2p_combine_experts_back")
                    ev = torch.cuda.Event()
                    ev.record(side)
            ev_back.append(ev)
        self._mark("experts")
        if self.profile:
            self._last_recv_ids = torch.cat(recv_ids)
        out = torch.empty(M, K, dtype=x.dtype, device=dev)
        for c, a in enumerate(arenas):
            t0, t1 = bounds[c], bounds[c + 1]
            main.wait_event(ev_back[c])
            _lib.check(lib.moe_p2p_wait(a["base"], W, 2, a["cap"], K, k, a["seq"], status, st_main), "moe_p2p_wait")
            if t1 > t0:  # NaN rows if any wait of this step gave up
                _lib.check(lib.moe_p2p_reduce(dt, a["base"], _ptr(tok_rows[c]), t1 - t0, K, k, W, a["cap"],
                                              _ptr(out[t0:t1]), status, st_main), "moe_p2p_reduce")
        self._mark("combine_back")
        if self._p2p_status is None:
            self._p2p_status = (torch.zeros(1, dtype=torch.int32).pin_memory(), torch.cuda.Event())
        host, ev = self._p2p_status
        host.copy_(status_word(dev), non_blocking=True)
        ev.record()
        if self.profile and self._marks:
            self.phase_log.append(self._marks)
        return out

    def close(self):
        self._p2p_release()
        self._ws = None
        self._ws_chunks = []
