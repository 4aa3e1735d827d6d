"""The C ABI from a plain C host (no Python): include/yufb200.h compiles as
C99, libyufb200.so links, and the host-only entry points work without a GPU
(tests/c/abi_check.c)."""

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs a C compiler")
def test_c_program_against_the_header_and_library(tmp_path):
    from yufmusicgen_b200 import _lib

    _lib.load()  # the library exists (built in tree)
    lib_dir = _lib.LIB_PATH.parent
    exe = tmp_path / "abi_check"
    cmd = ["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"), str(ROOT / "tests" / "c" / "abi_check.c"),
           "-L", str(lib_dir), "-lyufb200", f"-Wl,-rpath,{lib_dir}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert "c abi ok" in out.stdout
