"""The C ABI from a plain C caller: tests/c/abi_check.c includes only
include/b200mm.h, is compiled with the host C compiler against the built
library, and runs the calls that need no GPU."""

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
LIB = ROOT / "llms_b200" / "_lib"


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_c_caller_builds_and_passes(tmp_path):
    exe = tmp_path / "abi_check"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "c" / "abi_check.c"), "-L", str(LIB), "-lb200mm",
                    f"-Wl,-rpath,{LIB}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "abi_check: ok" in r.stdout
