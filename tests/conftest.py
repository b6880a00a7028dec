"""Shared test setup: the `gpu` marker, the package import and the checker."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import __graft_entry__  # noqa: E402

__graft_entry__.package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.lib()
    return oracle


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "golden.npz")))


@pytest.fixture(scope="session")
def ops():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from elffuss_engine_b200.ops import QuantOps
    return QuantOps(0)


_REPORT: dict = {}


@pytest.fixture(scope="session")
def parity_report():
    """Measured error ratios and token agreements, written as JSON at the end
    of the session to $EF_PARITY_REPORT when that is set (else only kept)."""
    return _REPORT


def pytest_sessionfinish(session, exitstatus):
    path = os.environ.get("EF_PARITY_REPORT")
    if path and _REPORT:
        import json
        with open(path, "w") as f:
            json.dump(_REPORT, f, indent=1, sort_keys=True)
