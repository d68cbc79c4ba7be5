"""The C ABI from C: tests/c/abi_host_calls.c is compiled as C99 against include/bsattn.h, linked
to the in-tree libbsattn.so and run (CPU only: the calls it makes need no GPU).  This checks
that the header is valid C and that a C caller links and gets the documented return codes."""
import os
import shutil
import subprocess

import pytest

from usagi_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_c_caller_builds_links_and_runs(tmp_path):
    lib = _lib.library_path()
    _lib.load()  # raises if the library is missing
    exe = tmp_path / "abi_host_calls"
    cmd = ["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "c", "abi_host_calls.c"), "-o", str(exe),
           "-L", str(lib.parent), "-l:" + lib.name, "-Wl,-rpath," + str(lib.parent)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().endswith("all ok"), r.stdout
