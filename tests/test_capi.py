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
