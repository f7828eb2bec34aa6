"""Shared test setup.

Markers: ``gpu`` = needs an sm_100 GPU (run with ``-m gpu`` on a B200);
everything else runs on the CPU (``-m "not gpu"``).
"""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def _ensure_built():
    from cube_awq_b200 import build as b
    b.build()
    b.build_torch_ext()
    import oracle
    oracle.build()


_ensure_built()


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    major, _ = torch.cuda.get_device_capability(0)
    if major != 10:
        pytest.fail(f"GPU tests need an sm_100 device, got sm_{major}x")
    return torch.device("cuda:0")
