"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device (a B200); everything else runs on CPU.
The product package lives in the `hesa-llm_b200/` directory, whose name is not
a Python identifier, so its directory is put on sys.path and its modules are
imported by their own names (`hesa_cuda`, ...).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "hesa-llm_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
