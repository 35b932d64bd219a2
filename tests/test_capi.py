"""CPU: the C-ABI library builds, loads without a GPU and exports every symbol of include/moe_b200.h.

Only host-side argument validation is called here (no kernel launches).
"""
import ctypes
import re

import pytest

from kernelswift_competition_submission_b200 import _lib, build

HEADER = build.ROOT / "include" / "moe_b200.h"


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def _declared():
    text = HEADER.read_text()
    return re.findall(r"MOE_API\s+[\w\s\*]+?\b(moe_\w+)\s*\(", text)


def test_header_declares_entry_points():
    names = _declared()
    assert {"moe_grouped_topk", "moe_align", "moe_fused_experts", "moe_fused_workspace_bytes"} <= set(names)


def test_every_declared_symbol_is_exported(lib):
    for name in _declared():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_no_extra_exports():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(build.OUT)], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert exported == set(_declared())


def test_status_strings(lib):
    assert _lib.status_string(0) == "ok"
    assert "workspace" in _lib.status_string(_lib.MOE_ERR_WORKSPACE)
    assert lib.moe_abi_version() >= 100


def test_grouped_topk_argument_validation(lib):
    f = lib.moe_grouped_topk
    # unsupported expert count / group layout / topk, all rejected on the host
    assert f(None, None, 4, 600, 8, 1, 8, 4, 0, 0, 1.0, None, None, None) == _lib.MOE_ERR_BAD_SHAPE
    assert f(None, None, 4, 256, 8, 1, 7, 4, 0, 0, 1.0, None, None, None) == _lib.MOE_ERR_BAD_SHAPE
    assert f(None, None, 4, 256, 200, 1, 8, 4, 0, 0, 1.0, None, None, None) == _lib.MOE_ERR_BAD_SHAPE
    assert f(None, None, 4, 256, 8, 1, 8, 4, 5, 0, 1.0, None, None, None) == _lib.MOE_ERR_INVALID_ARG
    assert f(None, None, -1, 256, 8, 1, 8, 4, 0, 0, 1.0, None, None, None) == _lib.MOE_ERR_INVALID_ARG
    # topk larger than the experts left after group masking (v0 would return -inf weights)
    assert f(None, None, 4, 16, 8, 1, 4, 1, 0, 0, 1.0, None, None, None) == _lib.MOE_ERR_BAD_SHAPE
    # empty batch: nothing to do, no launch
    assert f(None, None, 0, 256, 8, 1, 8, 4, 1, 1, 2.5, None, None, None) == _lib.MOE_OK
    # null pointers with work to do
    assert f(None, None, 4, 256, 8, 1, 8, 4, 1, 1, 2.5, None, None, None) == _lib.MOE_ERR_INVALID_ARG


def test_align_capacity(lib):
    assert lib.moe_align_capacity(0, 8, 128) == 1024  # 8 * 127 rounded up to a whole m-block
    assert lib.moe_align_capacity(262144, 256, 128) == 262144 + 256 * 127 + (-(262144 + 256 * 127)) % 128
    assert lib.moe_align_capacity(-1, 8, 128) == -1


def test_fused_argument_validation(lib):
    f = lib.moe_fused_experts
    p = ctypes.c_void_p(256)
    assert f(9, p, p, p, p, p, 4, 8, 2, 128, 64, p, p, 1 << 20, None, None) == _lib.MOE_ERR_UNSUPPORTED
    assert f(0, p, p, p, p, p, 4, 8, 2, 100, 64, p, p, 1 << 20, None, None) == _lib.MOE_ERR_BAD_SHAPE
    assert f(0, p, p, p, p, p, 4, 8, 2, 128, 96, p, p, 1 << 20, None, None) == _lib.MOE_ERR_BAD_SHAPE
    assert f(0, p, p, p, p, p, 0, 8, 2, 128, 64, p, p, 0, None, None) == _lib.MOE_OK
    assert f(0, None, p, p, p, p, 4, 8, 2, 128, 64, p, p, 1 << 20, None, None) == _lib.MOE_ERR_INVALID_ARG
    # misaligned pointer
    q = ctypes.c_void_p(258)
    assert f(0, q, p, p, p, p, 4, 8, 2, 128, 64, p, p, 1 << 20, None, None) == _lib.MOE_ERR_INVALID_ARG


def test_workspace_bytes_monotone(lib):
    a = lib.moe_fused_workspace_bytes(128, 256, 8, 7168, 2048)
    b = lib.moe_fused_workspace_bytes(4096, 256, 8, 7168, 2048)
    assert 0 < a < b
    assert lib.moe_fused_workspace_bytes(0, 0, 8, 7168, 2048) == 0


def test_p2p_arena_layout(lib):
    """The peer-memory arena layout: regions in order, 256-byte aligned, sized as documented."""
    world, cap, K, k = 8, 4096, 7168, 8
    offs = (ctypes.c_int64 * 9)()
    assert lib.moe_p2p_arena_offsets(world, cap, K, k, offs) == 0
    ready, disp, back, counts, rx, rid, rw, bx, total = list(offs)
    assert (ready, disp, back, counts) == (0, 4 * world, 8 * world, 12 * world)
    assert rx % 256 == 0 and rid % 256 == 0 and rw % 256 == 0 and bx % 256 == 0
    assert rid - rx >= world * cap * K * 2 and rw - rid >= world * cap * k * 4
    assert bx - rw >= world * cap * k * 4 and total - bx >= world * cap * K * 2
    assert lib.moe_p2p_arena_bytes(world, cap, K, k) == total
    # rejected shapes
    assert lib.moe_p2p_arena_bytes(65, cap, K, k) == -1
    assert lib.moe_p2p_arena_bytes(world, 0, K, k) == -1
    assert lib.moe_p2p_arena_offsets(world, cap, K, 33, offs) == _lib.MOE_ERR_INVALID_ARG


def test_router_argument_validation(lib):
    f = lib.moe_router_grouped_topk
    args = dict(dt=0, x=None, wg=None, b=None, M=4, E=256, K=7168, k=8, rn=1, ng=8, tg=4, sc=1, gm=1, s=2.5)

    def call(**kw):
        a = {**args, **kw}
        return f(a["dt"], a["x"], a["wg"], a["b"], a["M"], a["E"], a["K"], a["k"], a["rn"], a["ng"], a["tg"],
                 a["sc"], a["gm"], a["s"], None, None, None, None, None, None)

    assert call(E=128) == _lib.MOE_ERR_BAD_SHAPE        # the tile is all 256 experts
    assert call(K=7000) == _lib.MOE_ERR_BAD_SHAPE       # K in 64-wide steps
    assert call(ng=64) == _lib.MOE_ERR_BAD_SHAPE        # 4-expert groups are not whole lanes
    assert call(dt=2) == _lib.MOE_ERR_UNSUPPORTED       # fp32 operands
    assert call() == _lib.MOE_ERR_INVALID_ARG           # null pointers, caught before any launch
    assert call(M=0) == 0
    assert lib.moe_router_scratch_ints(257) == 3


def test_fp8_packed_row_format(lib):
    # K e4m3 codes + K / 128 fp32 scales, padded to 16 bytes
    assert lib.moe_fp8_row_bytes(7168) == 7168 + 224
    assert lib.moe_fp8_row_bytes(128) == 144
    assert lib.moe_fp8_row_bytes(512) == 528
    assert lib.moe_fp8_row_bytes(100) == -1 and lib.moe_fp8_row_bytes(0) == -1
    for K in range(128, 16385, 128):  # a packed row always fits a bf16 row slot of the p2p arena
        assert lib.moe_fp8_row_bytes(K) <= 2 * K and lib.moe_fp8_row_bytes(K) % 16 == 0


def test_fp8_rows_argument_validation(lib):
    f = lib.moe_fused_experts_fp8_rows
    rb = lib.moe_fp8_row_bytes(512)
    args = lambda M, stride, K, mc=0, fmt=0: f(None, stride, None, None, None, None, None, None, M, 8, 2, K, 256, fmt,
                                               None, None, 0, mc, None, None)
    assert args(4, rb - 16, 512) == _lib.MOE_ERR_INVALID_ARG     # pitch shorter than a packed row
    assert args(4, rb + 8, 512) == _lib.MOE_ERR_INVALID_ARG      # pitch not a multiple of 16
    assert args(4, rb, 500) == _lib.MOE_ERR_BAD_SHAPE            # K % 128 != 0
    assert args(4, rb, 512, -1) == _lib.MOE_ERR_INVALID_ARG      # negative grid limit
    assert args(0, rb, 512) == _lib.MOE_OK                       # no rows: nothing to do
    assert args(4, rb, 512) == _lib.MOE_ERR_INVALID_ARG          # null pointers
    assert args(4, rb, 512, 0, 2) == _lib.MOE_ERR_INVALID_ARG    # unknown scale format
    q = lib.moe_quantize_rows_fp8_packed
    assert q(0, None, 4, 500, None, 0, None) == _lib.MOE_ERR_BAD_SHAPE
    assert q(7, None, 4, 512, None, 0, None) == _lib.MOE_ERR_UNSUPPORTED
    assert q(0, None, 4, 512, None, 0, None) == _lib.MOE_ERR_INVALID_ARG
    assert q(0, None, 4, 512, None, 5, None) == _lib.MOE_ERR_INVALID_ARG  # unknown scale format
    # the EP pack and p2p dispatch take the packed rows only with K % 128 == 0
    pack = lib.moe_ep_pack
    assert pack(_lib.MOE_DTYPE_E4M3_ROW, None, None, None, 4, 520, 2, 4, 2, None, None, None, None, None,
                None) == _lib.MOE_ERR_BAD_SHAPE
