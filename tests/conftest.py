"""Shared fixtures.  `gpu` tests need a CUDA device and the in-tree liburb_moe.so; everything
else runs on the CPU (oracle, host logic, ABI surface)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and liburb_moe.so")


@pytest.fixture(scope="session")
def oracle():
    import urb_oracle
    urb_oracle.build()
    return urb_oracle


@pytest.fixture(scope="session")
def ctx():
    import urbilateria_b200 as urb
    return urb.default_context()
