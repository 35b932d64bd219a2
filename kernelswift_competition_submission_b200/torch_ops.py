"""PyTorch operator registrations over the C ABI: ``torch.ops.moe_b200.*``.

Importing the package registers these operators with ``torch.library``. Each one
calls the same ctypes entry point as the functional API in ``ops`` (the sm_100a
kernels of ``libmoe_b200.so``, no fallback), and each has a fake implementation that
only allocates outputs of the right shape and dtype, so shape propagation, meta
tensors and ``torch.compile`` graphs see the operators without running them:

    torch.ops.moe_b200.grouped_topk(hidden_states, gating_output, topk, renormalize,
                                    num_expert_group, topk_group, scoring_func,
                                    routed_scaling_factor, e_score_correction_bias)
        -> (topk_weights fp32 [M, topk], topk_ids int32 [M, topk])
        the launch of grouped_topk/v1/grouped_topk.py:210-235, rule of
        grouped_topk/v0/grouped_topk.py:91-132 (plus the bias / top-2 group sum)
    torch.ops.moe_b200.fused_moe(hidden_states, w1, w2, topk_weights, topk_ids)
        -> out [M, K] in the hidden dtype; the launches of fused_moe/v1/fused_moe.py:305-341,
        math of fused_moe/v0/fused_moe.py:141-167
    torch.ops.moe_b200.fused_moe_fp8(hidden_states, w1_q, w1_scale, w2_q, w2_scale,
                                     topk_weights, topk_ids, scale_format="") -> out bf16 [M, K]
        (scale_format "" decides from the weight scales: "ue8m0" when all are powers of two)
    torch.ops.moe_b200.moe_align(topk_ids, num_experts, block_m)
        -> (counts, block_start, sorted_pairs)  (sorted_pairs' length depends on the
        capacity rule; the fake uses the same formula)
    torch.ops.moe_b200.quantize_rows_fp8(x, scale_format="ue8m0") -> (q e4m3 [M, K], scales fp32 [M, K / 128])
    torch.ops.moe_b200.quantize_weights_fp8(w, scale_format="ue8m0")
        -> (q e4m3 [E, R, C], scales fp32 [E, R / 128, C / 128])

Every operator returns new tensors and writes none of its inputs (``mutates_args=()``).
"""

from typing import Optional

import torch
from torch import Tensor

from . import ops

_NS = "moe_b200"


@torch.library.custom_op(f"{_NS}::grouped_topk", mutates_args=())
def grouped_topk_op(hidden_states: Optional[Tensor], gating_output: Tensor, topk: int, renormalize: bool,
                    num_expert_group: int, topk_group: int, scoring_func: str = "softmax",
                    routed_scaling_factor: float = 1.0,
                    e_score_correction_bias: Optional[Tensor] = None) -> tuple[Tensor, Tensor]:
    return ops.grouped_topk(hidden_states, gating_output, topk, renormalize, num_expert_group, topk_group,
                            scoring_func, routed_scaling_factor, e_score_correction_bias)


@grouped_topk_op.register_fake
def _grouped_topk_fake(hidden_states, gating_output, topk, renormalize, num_expert_group, topk_group,
                       scoring_func="softmax", routed_scaling_factor=1.0, e_score_correction_bias=None):
    M = gating_output.shape[0]
    return (gating_output.new_empty(M, topk, dtype=torch.float32),
            gating_output.new_empty(M, topk, dtype=torch.int32))


@torch.library.custom_op(f"{_NS}::fused_moe", mutates_args=())
def fused_moe_op(hidden_states: Tensor, w1: Tensor, w2: Tensor, topk_weights: Tensor, topk_ids: Tensor) -> Tensor:
    return ops.fused_moe(hidden_states, w1, w2, topk_weights, topk_ids)


@fused_moe_op.register_fake
def _fused_moe_fake(hidden_states, w1, w2, topk_weights, topk_ids):
    return hidden_states.new_empty(hidden_states.shape)


@torch.library.custom_op(f"{_NS}::fused_moe_fp8", mutates_args=())
def fused_moe_fp8_op(hidden_states: Tensor, w1_q: Tensor, w1_scale: Tensor, w2_q: Tensor, w2_scale: Tensor,
                     topk_weights: Tensor, topk_ids: Tensor, scale_format: str = "") -> Tensor:
    return ops.fused_moe_fp8(hidden_states, w1_q, w1_scale, w2_q, w2_scale, topk_weights, topk_ids,
                             scale_format=scale_format or None)


@fused_moe_fp8_op.register_fake
def _fused_moe_fp8_fake(hidden_states, w1_q, w1_scale, w2_q, w2_scale, topk_weights, topk_ids, scale_format=""):
    return hidden_states.new_empty(hidden_states.shape, dtype=torch.bfloat16)


def _align_capacity(num_pairs: int, num_experts: int, block_m: int) -> int:
    # the rule of moe_align_capacity: every expert's segment rounded up to whole m-blocks
    cap = num_pairs + num_experts * (block_m - 1)
    return (cap + block_m - 1) // block_m * block_m


@torch.library.custom_op(f"{_NS}::moe_align", mutates_args=())
def moe_align_op(topk_ids: Tensor, num_experts: int, block_m: int = 128) -> tuple[Tensor, Tensor, Tensor]:
    counts, block_start, sorted_pairs = ops.moe_align(topk_ids, num_experts, block_m)
    return counts, block_start, sorted_pairs.clone()  # a fresh tensor, not a view of a larger one


@moe_align_op.register_fake
def _moe_align_fake(topk_ids, num_experts, block_m=128):
    cap = _align_capacity(topk_ids.numel(), num_experts, block_m)
    return (topk_ids.new_empty(num_experts, dtype=torch.int32), topk_ids.new_empty(num_experts + 1, dtype=torch.int32),
            topk_ids.new_empty(cap, dtype=torch.int32))


@torch.library.custom_op(f"{_NS}::quantize_rows_fp8", mutates_args=())
def quantize_rows_fp8_op(x: Tensor, scale_format: str = "ue8m0") -> tuple[Tensor, Tensor]:
    return ops.quantize_rows_fp8(x, scale_format)


@quantize_rows_fp8_op.register_fake
def _quantize_rows_fp8_fake(x, scale_format="ue8m0"):
    M, K = x.shape
    return x.new_empty(M, K, dtype=torch.float8_e4m3fn), x.new_empty(M, K // 128, dtype=torch.float32)


@torch.library.custom_op(f"{_NS}::quantize_weights_fp8", mutates_args=())
def quantize_weights_fp8_op(w: Tensor, scale_format: str = "ue8m0") -> tuple[Tensor, Tensor]:
    return ops.quantize_weights_fp8(w, scale_format)


@quantize_weights_fp8_op.register_fake
def _quantize_weights_fp8_fake(w, scale_format="ue8m0"):
    E, R, C = w.shape
    return w.new_empty(E, R, C, dtype=torch.float8_e4m3fn), w.new_empty(E, R // 128, C // 128, dtype=torch.float32)
