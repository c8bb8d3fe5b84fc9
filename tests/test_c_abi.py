"""The C ABI used from plain C: tests/c/abi_host_check.c is compiled with gcc against
include/orda_b200.h, linked to the built liborda_b200.so and run (host-only checks, no GPU)."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

from orda_ce_kernel import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_c_program_links_and_validates(tmp_path):
    lib = _native.LIB_PATH
    assert os.path.exists(lib), "build the library first"
    exe = tmp_path / "abi_host_check"
    libdir = os.path.dirname(lib)
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c", "abi_host_check.c"), "-o", str(exe),
                    "-L", libdir, "-l:" + os.path.basename(lib), "-Wl,-rpath," + libdir], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert "c abi ok" in out.stdout
