"""fused_moe drop-in: ``ModelNew`` for ``fused_moe/v1/fused_moe.py``.

Constructor, parameter names and shapes match the reference
(``fused_moe/v0/fused_moe.py:99-124``: ``w1 [E, 2I, H]``, ``w2 [E, H, I]``) so
the harness's ``load_state_dict`` weight copy works. The forward runs the
softmax top-k routing kernel and the sm_100a expert path (align, tcgen05
gate/up GEMM with fused SiLU*mul, tcgen05 down GEMM, top-k combine).
Repeated calls on the same input buffers replay a CUDA graph of the whole
forward (``graphs.GraphCache``: one launch instead of six kernels plus host work).
Weights cast to the hidden dtype are cached and refreshed when the parameter's
``_version`` or storage changes (the idea of ``fused_moe/v1/fused_moe.py:285-303``);
the cache is a plain attribute, not a registered buffer, so ``state_dict`` is
unchanged.
"""
import torch
import torch.nn as nn


def _bootstrap():
    import os
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(os.path.dirname(here))
    if root not in sys.path:
        sys.path.insert(0, root)
    import kernelswift_competition_submission_b200 as pkg

    return pkg


class ModelNew(nn.Module):
    def __init__(
        self,
        num_experts: int,
        top_k: int,
        hidden_size: int,
        intermediate_size: int,
        renormalize: bool = True,
    ):
        super().__init__()
        self.num_experts = num_experts
        self.top_k = top_k
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.renormalize = renormalize
        self.w1 = nn.Parameter(torch.empty(num_experts, 2 * intermediate_size, hidden_size))
        self.w2 = nn.Parameter(torch.empty(num_experts, hidden_size, intermediate_size))
        nn.init.normal_(self.w1, std=0.02)
        nn.init.normal_(self.w2, std=0.02)
        self._ops = _bootstrap()
        self._cache = None
        from kernelswift_competition_submission_b200.graphs import GraphCache

        self._graph = GraphCache(self._forward_eager)

    def _prepared_weights(self, dtype):
        # the parameter objects themselves are part of the key (held by the cache, so a new
        # parameter can never be mistaken for the old one at a reused address)
        key = (dtype, self.w1.device, self.w1.data_ptr(), self.w1._version, self.w2.data_ptr(), self.w2._version)
        if self._cache is None or self._cache[0] != key or self._cache[3] is not self.w1 or \
                self._cache[4] is not self.w2:
            with torch.no_grad():
                w1 = self.w1.detach().to(dtype).contiguous()
                w2 = self.w2.detach().to(dtype).contiguous()
            self._cache = (key, w1, w2, self.w1, self.w2)
        return self._cache[1], self._cache[2]

    def _forward_eager(self, hidden_states, router_logits, w1, w2):
        w, ids = self._ops.softmax_topk(router_logits, self.top_k, self.renormalize)
        return self._ops.fused_moe(hidden_states, w1, w2, w, ids)

    def forward(self, hidden_states: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        # repeated calls on the same buffers replay one CUDA graph of the whole forward
        w1, w2 = self._prepared_weights(hidden_states.dtype)
        return self._graph(hidden_states, router_logits, w1, w2)


def get_inputs():
    # hidden_states: [num_tokens, hidden_size] float16; router_logits: [num_tokens, num_experts] float32
    num_tokens, hidden_size, num_experts = 83, 128, 8
    hidden_states = torch.randn(num_tokens, hidden_size, dtype=torch.float16)
    router_logits = torch.randn(num_tokens, num_experts, dtype=torch.float32)
    return [hidden_states, router_logits]


def get_init_inputs():
    # num_experts, top_k, hidden_size, intermediate_size
    return [8, 2, 128, 64]
