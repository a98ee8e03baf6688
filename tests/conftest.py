"""Shared test set-up: import paths and the ``gpu`` marker.

Tests marked ``gpu`` need a CUDA device (a B200) and the in-tree CUDA library;
everything else runs on the CPU.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "comfyui-int4-convrot-rdna4_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the built CUDA library")
