"""grouped_topk drop-in: ``ModelNew`` for ``grouped_topk/v1/grouped_topk.py``.

Same constructor and forward signature as the reference's ModelNew
(``grouped_topk/v1/grouped_topk.py:187-235``) and v0 Model
(``grouped_topk/v0/grouped_topk.py:73-132``); the forward is one launch of the
warp-per-token sm_100a routing kernel in ``libmoe_b200.so``, launched directly: one
kernel, so a replayed CUDA graph (plus the copies that give each call fresh outputs) only
adds time here.
``get_inputs``/``get_init_inputs`` reproduce the task's CPU inputs
(``grouped_topk/v0/grouped_topk.py:135-148``).
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
        topk: int,
        renormalize: bool,
        num_expert_group: int,
        topk_group: int,
        scoring_func: str = "softmax",
        routed_scaling_factor: float = 1.0,
    ):
        super().__init__()
        self.topk = topk
        self.renormalize = renormalize
        self.num_expert_group = num_expert_group
        self.topk_group = topk_group
        self.scoring_func = scoring_func
        self.routed_scaling_factor = routed_scaling_factor
        self._ops = _bootstrap()

    def forward(self, hidden_states: torch.Tensor, gating_output: torch.Tensor):
        return self._ops.grouped_topk(
            hidden_states, gating_output, self.topk, self.renormalize, self.num_expert_group,
            self.topk_group, self.scoring_func, self.routed_scaling_factor)


def get_inputs():
    # hidden_states: [num_tokens, hidden_size] float16 (batch-size check only); gating_output fp32
    num_tokens, hidden_size, num_experts = 83, 7168, 256
    hidden_states = torch.randn(num_tokens, hidden_size, dtype=torch.float16)
    gating_output = torch.randn(num_tokens, num_experts, dtype=torch.float32)
    return [hidden_states, gating_output]


def get_init_inputs():
    # topk=8, renormalize=True, num_expert_group=8, topk_group=4
    return [8, True, 8, 4]
