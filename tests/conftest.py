"""pytest configuration: the ``gpu`` marker and shared helpers.

``-m "not gpu"`` runs here without a GPU (oracle pins, tracing/codegen,
NVRTC compiles, C-ABI exports, gloo multi-process host logic).  ``-m gpu``
runs on a B200 and calls the CUDA path through libthork_rt.so.
"""

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the CUDA path)")
