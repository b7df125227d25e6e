"""Test configuration.

``gpu``-marked tests need a B200 and the built CUDA library; everything else
runs on CPU (oracle against golden fixtures, host logic, gloo ranks, and the
C-ABI library's exported symbols).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "adaptive-precision-ascension_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built kernel library")
