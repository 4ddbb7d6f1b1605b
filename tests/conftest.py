"""pytest configuration: the `gpu` marker and the import path of the build.

Tests marked `gpu` need a CUDA device (a B200 for the tcgen05 kernels); the
rest run on CPU (oracle vs golden fixtures, host logic, C-ABI symbol checks,
gloo multi-process tests).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "radeon-igpu-forge_b200")
for p in (PKG, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
