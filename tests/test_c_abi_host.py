"""The public headers compile as plain C (C11, all warnings as errors) and a C program linked
against libpcu_b200.so runs the host-only entry points (tests/c_abi_host.c).  No GPU needed."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_c_host_builds_and_runs(tmp_path, provider):
    lib_dir = os.path.dirname(provider.LIBRARY)
    exe = tmp_path / "c_abi_host"
    build = subprocess.run(
        ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", os.path.join(ROOT, "include"),
         os.path.join(ROOT, "tests", "c_abi_host.c"), "-o", str(exe), "-L", lib_dir, "-lpcu_b200",
         f"-Wl,-rpath,{lib_dir}"],
        capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "c abi host ok" in run.stdout
