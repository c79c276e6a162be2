"""The C ABI from plain C: tests/c/abi_check.c is compiled as C11 with
-Wall -Wextra -Werror -pedantic against include/feml_b200.h, linked to
libfeml_b200.so and run (graph builder, planner, plan tensor IO through a
host-memory backend written in C, error reporting). No GPU needed."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_header_and_library_from_c(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    libdir = os.path.join(ROOT, "feml_b200")
    exe = tmp_path / "abi_check"
    subprocess.run([cc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic",
                    "-I", os.path.join(ROOT, "include"), os.path.join(ROOT, "tests", "c", "abi_check.c"),
                    "-L", libdir, "-lfeml_b200", "-Wl,-rpath," + libdir, "-o", str(exe)],
                   check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "ok"
