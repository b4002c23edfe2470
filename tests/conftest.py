import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "fluxrt-cpp_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")


@pytest.fixture(scope="session")
def cuda():
    """Skips unless a CUDA device is present; gpu-marked tests run only on the GPU box."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def pytest_terminal_summary(terminalreporter):
    """Achieved max-abs / mean-abs of each tolerance check next to its bar."""
    import parity_stats
    if not parity_stats.RECORDS:
        return
    tr = terminalreporter
    tr.section("measured errors (max-abs / mean-abs against the bar)")
    for test, what, mx, mn, bmx, bmn in parity_stats.RECORDS:
        tr.write_line(f"{test[:58]:58s} {what[:30]:30s} {mx:9.2e} / {mn:9.2e}   bar {bmx:.0e} / {bmn:.0e}")
