"""Shared test setup: import paths, the `gpu` marker, seeded case builders and the device fixture."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "onegpu-csharp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def device():
    import onegpu_cuda as og

    if og.device_count() < 1:
        pytest.fail("no CUDA device visible: the gpu tests need a B200")
    d = og.GpuDevice(0)
    yield d
    d.dispose()
