"""The C ABI on a B200 from plain C: tests/c/forward_backward.c (CUDA runtime,
no Python) is built with gcc against include/linearard_b200.h and run."""
import os
import shutil
import subprocess

import pytest

from linearard_b200 import _lib

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_c_program_runs_forward_and_backward(tmp_path):
    lib_dir = os.path.dirname(_lib.LIB_PATH)
    exe = tmp_path / "forward_backward"
    cmd = ["gcc", "-std=c11", "-O2", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"),
           os.path.join(ROOT, "tests", "c", "forward_backward.c"),
           "-L", lib_dir, "-llinearard_b200", f"-Wl,-rpath,{lib_dir}",
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}",
           "-lm", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.startswith("ok"), (r.stdout, r.stderr)
