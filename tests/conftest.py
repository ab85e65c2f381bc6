"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device (the B200 box); everything else runs on
the CPU-only build container (`pytest -m "not gpu"`).
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a)")
