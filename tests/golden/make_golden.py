"""Generate golden vectors by running the reference's own v0 modules.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py /path/to/kernelswift_competition_submission

It imports ``grouped_topk/v0/grouped_topk.py`` and ``fused_moe/v0/fused_moe.py``
from that checkout (never copied into this repository), runs their ``Model``
classes on CPU with seeded inputs, and writes the inputs and outputs as
``tests/golden/*.npz``. The seeding follows the reference harness
(``bench/auto_bench.py:378-409``): ``torch.manual_seed(42)`` before building the
model and again before ``get_inputs()``.

The committed ``.npz`` files are what the CPU tests use; this script is only
needed to regenerate them.
"""

from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _load(ref_root: Path, rel: str):
    path = ref_root / rel
    spec = importlib.util.spec_from_file_location(f"_golden_{path.stem}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _gt_case(gt_mod, name, M, E, init, seed, scale_inputs=1.0):
    topk, renorm, n_group, topk_group = init[:4]
    scoring = init[4] if len(init) > 4 else "softmax"
    scale = init[5] if len(init) > 5 else 1.0
    torch.manual_seed(seed)
    g = torch.randn(M, E, dtype=torch.float32) * scale_inputs
    h = torch.zeros(M, 1, dtype=torch.float16)
    model = gt_mod.Model(topk, renorm, n_group, topk_group, scoring, scale).eval()
    with torch.no_grad():
        w, ids = model(h, g)
    return dict(
        gating_output=g.numpy(), topk_weights=w.numpy(), topk_ids=ids.numpy(),
        topk=np.int64(topk), renormalize=np.int64(bool(renorm)), num_expert_group=np.int64(n_group),
        topk_group=np.int64(topk_group), scoring_func=np.array(scoring),
        routed_scaling_factor=np.float64(scale),
    )


def main(ref_root: str) -> None:
    ref = Path(ref_root)
    gt = _load(ref, "grouped_topk/v0/grouped_topk.py")
    fm = _load(ref, "fused_moe/v0/fused_moe.py")

    # --- grouped_topk: the reference task exactly (auto_bench seeding) ---
    torch.manual_seed(42)
    init = gt.get_init_inputs()
    model = gt.Model(*init).eval()
    torch.manual_seed(42)
    hidden, gating = gt.get_inputs()
    with torch.no_grad():
        w, ids = model(hidden, gating)
    np.savez_compressed(
        HERE / "grouped_topk_task.npz",
        gating_output=gating.numpy(), hidden_rows=np.int64(hidden.shape[0]),
        hidden_cols=np.int64(hidden.shape[1]), topk_weights=w.numpy(), topk_ids=ids.numpy(),
        topk=np.int64(init[0]), renormalize=np.int64(bool(init[1])),
        num_expert_group=np.int64(init[2]), topk_group=np.int64(init[3]),
        scoring_func=np.array("softmax"), routed_scaling_factor=np.float64(1.0),
    )

    # --- grouped_topk: more rule/shape combinations through the same v0 Model ---
    cases = {
        "grouped_topk_sigmoid_m128": (128, 256, [8, True, 8, 4, "sigmoid", 2.5], 42),
        "grouped_topk_ragged_m1": (1, 64, [4, False, 4, 2, "softmax", 1.0], 7),
        "grouped_topk_m37_e128": (37, 128, [6, True, 4, 2, "sigmoid", 1.5], 11),
        "grouped_topk_mixtral_m256": (256, 8, [2, True, 1, 1, "softmax", 1.0], 42),
        "grouped_topk_m300_e256_k8": (300, 256, [8, False, 8, 3, "softmax", 1.0], 5),
    }
    for name, (M, E, init_c, seed) in cases.items():
        np.savez_compressed(HERE / f"{name}.npz", **_gt_case(gt, name, M, E, init_c, seed))

    # --- fused_moe: the reference task exactly (fp16) plus the fp32 run of the same v0 ---
    torch.manual_seed(42)
    finit = fm.get_init_inputs()
    fmodel = fm.Model(*finit).eval()
    torch.manual_seed(42)
    hs, logits = fm.get_inputs()
    with torch.no_grad():
        out16 = fmodel(hs, logits)
        w1h = fmodel.w1.detach().to(torch.float16)
        w2h = fmodel.w2.detach().to(torch.float16)
        # fp32 run of the same v0 code on the fp16-rounded operands
        fmodel32 = fm.Model(*finit).eval()
        fmodel32.w1.data.copy_(w1h.float())
        fmodel32.w2.data.copy_(w2h.float())
        out32 = fmodel32(hs.float(), logits)
    np.savez_compressed(
        HERE / "fused_moe_task.npz",
        hidden_states=hs.numpy(), router_logits=logits.numpy(), w1=w1h.numpy(), w2=w2h.numpy(),
        out_fp16=out16.numpy(), out_fp32=out32.numpy(),
        num_experts=np.int64(finit[0]), top_k=np.int64(finit[1]),
        hidden_size=np.int64(finit[2]), intermediate_size=np.int64(finit[3]),
    )

    # --- fused_moe: a small fp32 case with a ragged token count ---
    torch.manual_seed(3)
    E, k, H, I, M = 4, 2, 128, 64, 17
    small = fm.Model(E, k, H, I).eval()
    x = torch.randn(M, H, dtype=torch.float32)
    lg = torch.randn(M, E, dtype=torch.float32)
    with torch.no_grad():
        o = small(x, lg)
    np.savez_compressed(
        HERE / "fused_moe_small_fp32.npz",
        hidden_states=x.numpy(), router_logits=lg.numpy(), w1=small.w1.detach().numpy(),
        w2=small.w2.detach().numpy(), out_fp32=o.numpy(), num_experts=np.int64(E), top_k=np.int64(k),
        hidden_size=np.int64(H), intermediate_size=np.int64(I),
    )
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
