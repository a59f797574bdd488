import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (run on the B200 box with -m gpu)")


def pytest_collection_modifyitems(config, items):
    # Without a GPU, -m gpu tests would only fail; mark them skipped with a reason
    # unless the caller explicitly selected them (then they must run and fail loudly).
    import torch
    selected = config.getoption("-m") or ""
    if torch.cuda.is_available() or "gpu" in selected and "not gpu" not in selected:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
