import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _no_device_wait_errors(request):
    """After every GPU test: no kernel of the library may have given up on a
    bounded on-chip wait (such a kernel ends with partial output, so a test
    that passed on it would prove nothing)."""
    yield
    if "gpu" not in request.keywords:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from lightserve_b200 import check_device_errors

    check_device_errors(reset=True)
