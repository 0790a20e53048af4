"""The C ABI from plain C: tests/c/abi_check.c is compiled with gcc against
include/linearard_b200.h, linked to the built liblinearard_b200.so and run
(host-only calls: version, status strings, workspace sizes, validation)."""
import os
import shutil
import subprocess

import pytest

from linearard_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_c_program_against_the_header_and_library(tmp_path):
    lib_dir = os.path.dirname(_lib.LIB_PATH)
    exe = tmp_path / "abi_check"
    cmd = ["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "c", "abi_check.c"), "-L", lib_dir,
           "-llinearard_b200", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", (r.stdout, r.stderr)
