"""Shared test setup.

* registers the ``gpu`` marker: tests that need a B200 carry it; the CPU suite
  runs with ``-m "not gpu"``;
* puts ``oracle/`` (the CPU checker) and the package directory on sys.path.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", "demucs-wgpu_b200", "tests"):
    path = os.path.join(ROOT, sub)
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle

    oracle.lib()
    return oracle
