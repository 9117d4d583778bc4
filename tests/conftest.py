"""Shared pytest setup: the `gpu` marker, repo-root imports and the CUDA context fixture."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; runs the CUDA kernels through the C ABI")


@pytest.fixture(scope="session")
def ctx():
    import torch

    from aihost_b200.ops import Context

    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    c = Context(0)
    yield c
    c.close()
