"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs the CPU suite (oracle vs golden vectors, host logic, C-ABI
exports); `-m gpu` runs the CUDA parity tests on a B200.
"""

import json
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import oxiref
    oxiref.lib()
    return oxiref


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "composed_small.npz")))


@pytest.fixture(scope="session")
def native():
    from oxitorch_b200 import _native
    return _native.load(require_device=True)


def pytest_sessionfinish(session, exitstatus):
    """With $OXC_STRICT_REPORT set, writes every parity check's count of
    elements beyond the bare tolerance (tests/parity.py STRICT_LOG) there."""
    path = os.environ.get("OXC_STRICT_REPORT")
    if not path:
        return
    try:
        import parity
    except ImportError:
        return
    with open(path, "w") as f:
        json.dump(parity.STRICT_LOG, f, indent=0)
