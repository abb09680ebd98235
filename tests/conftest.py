"""Shared test setup: the ``gpu`` marker, the in-tree library build, seeded inputs on the device."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: imports vLLM or runs large cases")
    from qwen_a100_fastpath_b200.build import build_library, needs_build
    if needs_build():
        build_library()


def cuda_ok() -> bool:
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    except Exception:  # noqa: BLE001
        return False


@pytest.fixture(scope="session")
def dev():
    import torch
    if not cuda_ok():
        pytest.fail("GPU test run without a B200 (compute capability 10.0) visible")
    return torch.device("cuda", 0)


def to_dev_bf16(bits: np.ndarray, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def from_dev_bf16(t) -> np.ndarray:
    import torch
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)
