"""Test set-up: import paths and the ``gpu`` marker.

``-m "not gpu"`` runs on any machine (oracle against the golden fixtures, host logic, the C-ABI library's exports);
``-m gpu`` needs an sm_100 GPU and the built ``libt2w_b200.so`` and compares the CUDA path with the oracle.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "minicpm-o-4.5-single-gpu-engine_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(ROOT, "tests", "golden")
