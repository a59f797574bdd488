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


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Print how close every bf16 output (h_in, dx) came to its reference:
    elements bit-equal, within 1 ulp, needing the fp32 floor, worst ulps."""
    try:
        from tests._gpu import BF16_REPORT
    except Exception:   # noqa: BLE001 - the GPU helpers were never imported
        return
    if not BF16_REPORT:
        return
    tr = terminalreporter
    tr.write_sep("-", "bf16 outputs vs reference (1 ulp + 2^-18 sum|terms| bar)")
    tr.write_line(f"{'case':34s} {'out':5s} {'elements':>10s} {'exact':>7s} {'<=1ulp':>7s} "
                  f"{'floor':>6s} {'worst':>6s} {'worst<=1ulp-part':>6s}")
    for tag, name, st in BF16_REPORT:
        n = max(st["n"], 1)
        tr.write_line(f"{tag[:34]:34s} {name:5s} {st['n']:10d} {st['exact'] / n:7.4f} {st['within_ulp'] / n:7.4f} "
                      f"{st['floor_needed']:6d} {st['worst_ulps']:6.1f} {st['worst_ulps_no_floor']:6.2f}")
