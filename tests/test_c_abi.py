"""The C ABI from plain C: tests/c_abi/c_caller.c is compiled with gcc -std=c99 against
include/fa2_sm100.h, linked to the built libfa2_sm100.so and run. It needs no GPU: it only uses
the host-side entry points (validation, workspace sizing, configuration, error strings) and the
ABI version / struct-size handshake a C, Go (cgo) or Rust (FFI) binding would perform."""

import os
import shutil
import subprocess

import pytest

from fa2 import _lib

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_plain_c_caller(tmp_path):
    _lib.lib()  # the library is built and loadable
    lib_dir = os.path.dirname(_lib.LIB_PATH)
    exe = tmp_path / "c_caller"
    cmd = ["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(REPO, "include"),
           os.path.join(HERE, "c_abi", "c_caller.c"), "-o", str(exe), "-L", lib_dir, "-l:libfa2_sm100.so",
           f"-Wl,-rpath,{lib_dir}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "ALL OK" in run.stdout
