"""ctypes binding of the C-ABI library ``libmoe_b200.so`` (declared in include/moe_b200.h).

The library is built in-tree by ``kernelswift_competition_submission_b200.build``.
There is no fallback: if the library is missing or fails to load, every op
raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_NAME = "libmoe_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

MOE_OK = 0
MOE_ERR_INVALID_ARG = 1
MOE_ERR_BAD_SHAPE = 2
MOE_ERR_UNSUPPORTED = 3
MOE_ERR_NOT_SM100 = 4
MOE_ERR_WORKSPACE = 5
MOE_ERR_CUDA = 6
MOE_ERR_TIMEOUT = 7
MOE_ERR_SCRATCH_LIMIT = 8
MOE_NOALLOC_MAX_EXPERTS = 1024

MOE_SCORING_SOFTMAX = 0
MOE_SCORING_SIGMOID = 1
MOE_GROUP_SCORE_MAX = 0
MOE_GROUP_SCORE_TOP2_SUM = 1
MOE_DTYPE_BF16 = 0
MOE_DTYPE_FP16 = 1
MOE_DTYPE_FP32 = 2
MOE_DTYPE_E4M3_ROW = 3
MOE_FP8_SCALE_FP32 = 0
MOE_FP8_SCALE_UE8M0 = 1

_c_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); must match include/moe_b200.h exactly
SIGNATURES = {
    "moe_status_string": (ctypes.c_char_p, [_i32]),
    "moe_abi_version": (_i32, []),
    "moe_check_device": (_i32, []),
    "moe_grouped_topk": (_i32, [_c_p, _c_p, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _f32, _c_p, _c_p, _c_p]),
    "moe_align_capacity": (_i64, [_i64, _i32, _i32]),
    "moe_align": (_i32, [_c_p, _i64, _i32, _i32, _c_p, _c_p, _c_p, _i64, _c_p, _c_p]),
    "moe_align_noalloc": (_i32, [_c_p, _i64, _i32, _i32, _c_p, _c_p, _c_p, _i64, _c_p]),
    "moe_fused_workspace_bytes": (_sz, [_i64, _i32, _i32, _i32, _i32]),
    "moe_fused_experts": (_i32, [_i32, _c_p, _c_p, _c_p, _c_p, _c_p, _i64, _i32, _i32, _i32, _i32, _c_p, _c_p, _sz,
                                 _c_p, _c_p]),
    "moe_expert_align_gather": (_i32, [_i32, _c_p, _c_p, _i64, _i32, _i32, _i32, _i32, _c_p, _sz, _c_p]),
    "moe_expert_align": (_i32, [_c_p, _i64, _i32, _i32, _i32, _i32, _c_p, _sz, _c_p]),
    "moe_expert_gemm1_gather": (_i32, [_i32, _c_p, _c_p, _i64, _i32, _i32, _i32, _i32, _c_p, _sz, _c_p, _i32,
                                       _c_p]),
    "moe_expert_gemm1": (_i32, [_i32, _c_p, _i64, _i32, _i32, _i32, _i32, _c_p, _sz, _c_p, _i32, _c_p]),
    "moe_expert_gemm2": (_i32, [_i32, _c_p, _i64, _i32, _i32, _i32, _i32, _c_p, _sz, _c_p, _i32, _c_p]),
    "moe_expert_gemm2_combine": (_i32, [_i32, _c_p, _c_p, _c_p, _i64, _i32, _i32, _i32, _i32, _c_p, _c_p, _sz, _c_p,
                                        _i32, _c_p]),
    "moe_expert_combine": (_i32, [_i32, _c_p, _c_p, _i64, _i32, _i32, _i32, _i32, _c_p, _c_p, _sz, _c_p]),
    "moe_quantize_rows_fp8": (_i32, [_i32, _c_p, _i64, _i32, _c_p, _c_p, _i32, _c_p]),
    "moe_quantize_blocks_fp8": (_i32, [_i32, _c_p, _i64, _i32, _i32, _c_p, _c_p, _i32, _c_p]),
    "moe_fused_workspace_bytes_fp8": (_sz, [_i64, _i32, _i32, _i32, _i32]),
    "moe_fused_experts_fp8": (_i32, [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _i64, _i32, _i32, _i32, _i32, _i32,
                                     _c_p, _c_p, _sz, _c_p, _c_p]),
    "moe_fp8_row_bytes": (_i64, [_i32]),
    "moe_quantize_rows_fp8_packed": (_i32, [_i32, _c_p, _i64, _i32, _c_p, _i32, _c_p]),
    "moe_fused_experts_fp8_rows": (_i32, [_c_p, _i64, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _i64, _i32, _i32, _i32, _i32,
                                          _i32, _c_p, _c_p, _sz, _i32, _c_p, _c_p]),
    "moe_ep_send_capacity": (_i64, [_i64, _i32, _i32]),
    "moe_ep_plan": (_i32, [_c_p, _i64, _i32, _i32, _i32, _c_p, _c_p, _c_p, _c_p]),
    "moe_ep_pack": (_i32, [_i32, _c_p, _c_p, _c_p, _i64, _i32, _i32, _i32, _i32, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p]),
    "moe_router_scratch_ints": (_i64, [_i64]),
    "moe_router_grouped_topk": (_i32, [_i32, _c_p, _c_p, _c_p, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32,
                                       _f32, _c_p, _c_p, _c_p, _c_p, _c_p, _c_p]),
    "moe_p2p_arena_bytes": (_i64, [_i32, _i64, _i32, _i32]),
    "moe_p2p_arena_offsets": (_i32, [_i32, _i64, _i32, _i32, _c_p]),
    "moe_p2p_alloc": (_i32, [_i32, _i64, _i32, _i32, _c_p, _c_p]),
    "moe_p2p_open": (_i32, [_c_p, _c_p]),
    "moe_p2p_close": (_i32, [_c_p]),
    "moe_p2p_free": (_i32, [_c_p]),
    "moe_p2p_signal": (_i32, [_c_p, _i32, _i32, _i32, _i64, _i32, _i32, ctypes.c_uint32, _c_p, _c_p]),
    "moe_p2p_wait": (_i32, [_c_p, _i32, _i32, _i64, _i32, _i32, ctypes.c_uint32, _c_p, _c_p]),
    "moe_p2p_dispatch": (_i32, [_i32, _c_p, _c_p, _c_p, _i64, _i32, _i32, _i32, _i32, _i32, _i64, _c_p, _c_p,
                                ctypes.c_uint32, _c_p, _c_p, _c_p, _c_p]),
    "moe_p2p_combine_experts_back": (_i32, [_i32, _c_p, _i32, _i32, _i32, _i32, _i32, _i32, _i64, _c_p, _c_p,
                                            ctypes.c_uint32, _c_p, _c_p, _c_p]),
    "moe_p2p_expert_gemm2_return": (_i32, [_i32, _c_p, _c_p, _sz, _i32, _i32, _i32, _i32, _i32, _i32, _i64, _c_p,
                                           _c_p, ctypes.c_uint32, _c_p, _c_p, _i32, _c_p]),
    "moe_p2p_copy_recv_ids": (_i32, [_c_p, _i32, _i64, _i32, _i32, _c_p, _c_p]),
    "moe_p2p_combine_back": (_i32, [_i32, _c_p, _i32, _i32, _i32, _i32, _i64, _c_p, _c_p, ctypes.c_uint32, _c_p,
                                    _c_p, _c_p]),
    "moe_p2p_reduce": (_i32, [_i32, _c_p, _c_p, _i64, _i32, _i32, _i32, _i64, _c_p, _c_p, _c_p]),
    "moe_ep_plan_mapped": (_i32, [_c_p, _i64, _i32, _i32, _c_p, _i32, _c_p, _c_p, _c_p, _c_p]),
    "moe_ep_pack_mapped": (_i32, [_i32, _c_p, _c_p, _c_p, _i64, _i32, _i32, _i32, _c_p, _i32, _c_p, _c_p, _c_p, _c_p,
                                  _c_p, _c_p]),
    "moe_ep_combine": (_i32, [_i32, _c_p, _c_p, _i64, _i32, _i32, _c_p, _c_p]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load the library once; raise RuntimeError when it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("MOE_B200_LIB", LIB_PATH))
    if not path.is_file():
        raise RuntimeError(
            f"{path} is missing: build it with `python -m kernelswift_competition_submission_b200.build` "
            "(the B200 MoE ops have no CPU or Python fallback)")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def status_string(code: int) -> str:
    return load().moe_status_string(code).decode()


def check(code: int, what: str) -> None:
    if code != MOE_OK:
        raise RuntimeError(f"{what} failed: {status_string(code)} (status {code})")
