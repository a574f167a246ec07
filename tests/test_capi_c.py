"""The public header compiles as C99 and as C++ without warnings, and a C
program linked against the built library makes host-side calls through it
(tests/c_abi_check.c; no GPU needed)."""
import os
import shutil
import subprocess

import pytest

from conftest import REPO

INC = os.path.join(REPO, "include")
LIB_DIR = os.path.join(REPO, "flagos-kernel-gen_b200", "lib")
SRC = os.path.join(REPO, "tests", "c_abi_check.c")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not installed")
def test_c_program_links_and_calls_the_library(pkg, tmp_path):
    exe = str(tmp_path / "c_abi_check")
    cc = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", INC, SRC, "-o", exe,
                         "-L", LIB_DIR, "-lw4a8moe", f"-Wl,-rpath,{LIB_DIR}"], capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0 and run.stdout.strip() == "ok", (run.returncode, run.stdout, run.stderr)


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not installed")
def test_header_compiles_as_cpp(tmp_path):
    src = tmp_path / "h.cpp"
    src.write_text('#include "w4a8moe.h"\nint (*probe)(void) = &w4a8_abi_version;\n')
    cc = subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", INC, "-c", str(src),
                         "-o", str(tmp_path / "h.o")], capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
