"""pytest configuration: the `gpu` marker and repository imports.

`-m "not gpu"` runs on any machine: the oracle against the reference's golden
vectors, the synthetic formats, and the C-ABI library's exports. `-m gpu`
runs the parity tests through the C ABI on an sm_100 device.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) device")


@pytest.fixture(scope="session")
def cuda_lib():
    """The backend bound to cuda:0 (gpu tests only)."""
    import warp_b200 as wb
    from warp_b200 import build
    build.build()
    name = wb.init(0)
    yield wb
    wb.shutdown()
