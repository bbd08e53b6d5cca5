"""Build recipe for ``libthork_rt.so``, the native half of thork_b200.

The library is compiled in-tree with nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``); nvcc cross-compiles without a
GPU.  Object files are rebuilt when a source or header is newer.

Usage: ``python -m thork_b200.build [--force] [--verbose]``.
"""

import os
import shutil
import subprocess
import sys
from typing import List

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
LIB_DIR = os.path.join(PKG_DIR, "lib")
OBJ_DIR = os.path.join(PKG_DIR, "_build")
LIB_PATH = os.path.join(LIB_DIR, "libthork_rt.so")

SOURCES = ["thork_rt.cu", "kernels.cu", "staging.cu", "multicast.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def find_nvcc() -> str:
    for env in ("CUDA_HOME", "CUDA_PATH"):
        root = os.environ.get(env)
        if root and os.path.isfile(os.path.join(root, "bin", "nvcc")):
            return os.path.join(root, "bin", "nvcc")
    found = shutil.which("nvcc")
    if found:
        return found
    if os.path.isfile("/usr/local/cuda/bin/nvcc"):
        return "/usr/local/cuda/bin/nvcc"
    raise RuntimeError("nvcc not found: set CUDA_HOME")


def _headers() -> List[str]:
    out = [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    for root, _dirs, files in os.walk(CSRC):
        out += [os.path.join(root, f) for f in files if f.endswith((".h", ".cuh"))]
    return out


def _stale(target: str, deps: List[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile libthork_rt.so if any source changed; return its path."""
    nvcc = find_nvcc()
    os.makedirs(LIB_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    headers = _headers()
    common = [
        nvcc, *ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17",
        "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        "-I", INCLUDE, "-I", CSRC,
        "--expt-relaxed-constexpr",
    ]
    objs = []
    for src in SOURCES:
        src_path = os.path.join(CSRC, src)
        obj = os.path.join(OBJ_DIR, src.replace(".cu", ".o"))
        objs.append(obj)
        if force or _stale(obj, [src_path] + headers):
            cmd = common + ["-c", src_path, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB_PATH, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", LIB_PATH, *objs, "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print(LIB_PATH)
