"""Pytest configuration: the ``gpu`` marker and shared fixtures.

``-m "not gpu"`` runs everywhere (oracle pins, host logic, C-ABI exports,
gloo multi-process tests); ``-m gpu`` needs a B200 and exercises the CUDA
library through the public API / C ABI.
"""

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
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running case")


@pytest.fixture(scope="session")
def sas_lib():
    from dsv4_b200 import build, _lib

    build.build()
    return _lib.lib()
