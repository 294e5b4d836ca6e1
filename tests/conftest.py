"""Shared pytest setup: markers and import paths.

`-m gpu` tests need a B200 and call the CUDA library through its C ABI;
everything else runs on the CPU (oracle against golden vectors, host logic,
library loading and symbol exports).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "voxcpm-cpp_b200")
for p in (ROOT, PKG, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
