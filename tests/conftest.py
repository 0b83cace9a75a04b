import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multigpu: needs at least 2 GPUs")
    config.addinivalue_line("markers", "slow: long-running (full-size model) test")


def _have_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def krlib():
    """The built libkernrelay.so (built in-tree if missing or stale)."""
    from kernrelay_b200 import build
    if not os.environ.get("KRB_NO_BUILD"):
        try:
            build.build()
        except RuntimeError:
            if not build.LIB.exists():
                raise
    from kernrelay_b200 import _lib
    return _lib


@pytest.fixture(scope="session")
def cuda(krlib):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    return torch.device("cuda:0")
