"""The strict MSE walk's round planner (fusion-pcu_b200/csrc/mse_walk_plan.h, the code the device
walker runs) built for the host and checked on two million random rounds: the planned maps follow
one another from the walk's position without a gap, stay in front of the stop, leave out a failed
map, are each of the coarsest level their position allows, and reach the stop unless the round is
full (tests/walk_plan_check.cpp).  No GPU needed."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_walk_plan_host_check(tmp_path):
    exe = tmp_path / "walk_plan_check"
    build = subprocess.run(
        ["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-I",
         os.path.join(ROOT, "fusion-pcu_b200", "csrc"), os.path.join(ROOT, "tests", "walk_plan_check.cpp"), "-o",
         str(exe)],
        capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "walk plan ok" in run.stdout
