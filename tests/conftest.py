import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden_dir():
    return GOLDEN


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a CUDA device")
    from kernelswift_competition_submission_b200 import _lib

    lib = _lib.load()
    code = lib.moe_check_device()
    if code != 0:
        pytest.fail(f"device is not sm_100: {_lib.status_string(code)}")
    return torch.device("cuda", 0)
