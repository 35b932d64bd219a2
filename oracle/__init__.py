"""CPU oracle for the MoE-layer hot path (grouped_topk routing -> fused_moe experts).

This package is TEST INFRASTRUCTURE. It is a numpy restatement of the
reference's PyTorch ``v0`` implementations and exists only to check the CUDA
path:

* ``tests/`` use it as the parity checker,
* ``__graft_entry__.smoke()`` uses it to check one small GPU call,
* ``bench.py`` times it as the ``cpu_baseline`` leg and as the ``--impl
  reference`` arm (the reference itself is Python/Triton and cannot travel to
  the GPU host).

The product path (``kernelswift_competition_submission_b200``) never imports
this package and never falls back to it.

Pinning: every function is checked against golden vectors produced by running
the reference's own ``v0`` modules in the build container
(``tests/golden/make_golden.py`` -> ``tests/golden/*.npz``). Rules that the
reference does not implement (``e_score_correction_bias``, the per-group top-2
sum, FP8 block quantisation) are documented extensions of ``v0`` and are
parity-unpinned by the reference; they reduce to ``v0`` bit-exactly when the
extension is switched off, which the tests check.
"""

from .grouped_topk import grouped_topk_ref, softmax_topk_ref  # noqa: F401
from .fused_moe import (  # noqa: F401
    moe_align_ref,
    moe_experts_ref,
    moe_experts_rows_ref,
    fused_moe_layer_ref,
    silu,
)
