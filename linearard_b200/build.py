"""Build ``liblinearard_b200.so`` in-tree with nvcc for sm_100a.

    python -m linearard_b200.build          # or __graft_entry__.build()

The library is one translation unit (``csrc/liblinearard_b200.cu``) compiled to
``linearard_b200/_lib/liblinearard_b200.so``.  nvcc cross-compiles, so this runs
on machines without a GPU.  The CUDA runtime is linked statically; the driver
entry point for TMA descriptors is looked up at run time, so the library
needs no libcuda at link time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT_DIR = os.path.join(PKG, "_lib")
LIB_NAME = "liblinearard_b200.so"
LIB_PATH = os.path.join(OUT_DIR, LIB_NAME)

SOURCES = ["liblinearard_b200.cu", "lkl_api.cu", "lkl_generic.cu", "lkl_sm100.cu", "lkl_noalloc.cu",
           "lkl_common.cuh", "sm100_ptx.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build liblinearard_b200")


def _stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, s) for s in SOURCES] + [os.path.join(ROOT, "include", "linearard_b200.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if it is missing or older than its sources."""
    if not force and not _stale():
        return LIB_PATH
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"),
           "-o", tmp, os.path.join(CSRC, "liblinearard_b200.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stdout + res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
