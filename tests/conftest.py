import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import __graft_entry__ as ge  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session")
def pkg():
    return ge.package()


@pytest.fixture(scope="session")
def oracle():
    o = ge.oracle()
    o.build()
    return o


@pytest.fixture(scope="session")
def wl(pkg):
    from mlir_flashattention_b200 import workloads

    return workloads
