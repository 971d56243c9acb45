"""The C ABI from C: tests/c_abi_consumer.c compiles as strict C99 against include/ptxstd.h,
links libptxstd.so and runs its GPU-free checks (no GPU needed)."""

import os
import shutil
import subprocess

import pytest

from conftest import ROOT


def test_c99_consumer(ptxstd_lib):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    libdir = os.path.join(ROOT, "ptx-std_b200")
    out_dir = os.path.join(libdir, "_build")
    os.makedirs(out_dir, exist_ok=True)
    exe = os.path.join(out_dir, "c_abi_consumer")
    subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic",
                    "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c_abi_consumer.c"), "-o", exe,
                    "-L", libdir, "-lptxstd", "-Wl,-rpath," + libdir], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr
