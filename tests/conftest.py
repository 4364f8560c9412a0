import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
TESTS = os.path.dirname(os.path.abspath(__file__))
if TESTS not in sys.path:
    sys.path.insert(0, TESTS)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and the built CUDA library")
    config.addinivalue_line("markers", "slow: long-running case")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except Exception:
        have_gpu = False
    if have_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Near-ties exempted by the reference-arithmetic parity level (GPU runs)."""
    try:
        from helpers import NEAR_TIES
    except Exception:
        return
    if not NEAR_TIES:
        return
    checks = len(NEAR_TIES)
    ties = sum(t for _, t, _ in NEAR_TIES)
    cands = sum(n for _, _, n in NEAR_TIES)
    worst = max(NEAR_TIES, key=lambda x: x[1])
    terminalreporter.write_line(
        f"near-ties exempted at the selection boundary: {ties} of {cands} candidates over {checks} parity "
        f"checks (most in one check: {worst[1]} of {worst[2]}, {worst[0]})")
