"""pytest configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a CUDA device and the built library; everything else
runs on CPU.  The repository root and the package folder are put on sys.path so
that `oracle`, `saccade_core` and `np_restatement` import without installation.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "saccade-x2_b200"), os.path.dirname(os.path.abspath(__file__))):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built CUDA library")
