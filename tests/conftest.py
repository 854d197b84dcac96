"""Test configuration: markers and import paths.

``-m gpu`` tests need a CUDA device (a B200) and call the CUDA library through
its C ABI; everything else runs on the CPU (oracle vs golden fixtures, host
logic, the C-ABI symbol table, gloo multi-process logic).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "polar-flash_b200")
for p in (ROOT, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a) and the built CUDA library")
