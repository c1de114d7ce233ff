"""Shared pytest configuration.

Markers: `gpu` marks tests that need a CUDA device (run with `-m gpu` on a
B200); everything else runs on the CPU. Mirrors the reference suite's
per-test seeding (tests/conftest.py:8-13 there).
"""
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200 / sm_100a)")


def pytest_sessionfinish(session, exitstatus):
    """Writes the parity counts the GPU tests recorded (tests/parity.py) to
    the file named by SSA_PARITY_COUNTS, if set and anything was recorded."""
    path = os.environ.get("SSA_PARITY_COUNTS")
    if not path:
        return
    import json
    import parity
    if not parity.COUNTS:
        return
    with open(path, "w") as f:
        json.dump({"band": {"hash_near_zero": 1e-6, "rescore_tie_rel": 64 * 2.0 ** -24},
                   "cases": parity.COUNTS}, f, indent=1, sort_keys=True)


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(42)
    yield


@pytest.fixture
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
