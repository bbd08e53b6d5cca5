"""pytest configuration: the ``gpu`` marker and shared helpers.

``-m "not gpu"`` runs here without a GPU (oracle pins, tracing/codegen,
NVRTC compiles, C-ABI exports, gloo multi-process host logic).  ``-m gpu``
runs on a B200 and calls the CUDA path through libthork_rt.so.
"""

import os
import sys
import tempfile

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

# keep the NVRTC cubin cache and temporary files of the test run inside the
# checkout (in the git-ignored build folder)
_SCRATCH = os.path.join(REPO, "thork_b200", "_build", "test_scratch")
os.makedirs(os.path.join(_SCRATCH, "tmp"), exist_ok=True)
os.environ.setdefault("THORK_CACHE_DIR", os.path.join(_SCRATCH, "nvrtc_cache"))
tempfile.tempdir = os.path.join(_SCRATCH, "tmp")


# byte-for-byte copies of the reference's test files, run only through
# test_gpu_reference_suite.py (they import `thork`, which that test aliases)
collect_ignore = ["_reference_suite"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the CUDA path)")
