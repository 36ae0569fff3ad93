"""bench.py's reference arm, which needs no GPU: it prints the one JSON line the benchmark
contract asks for, with the GPU arm's metric and workload, a single-thread cpu_baseline and an e2e
object with no host copies; under torchrun only rank 0 prints it."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, env_extra=None):
    env = dict(os.environ)
    for key in ("RANK", "LOCAL_RANK", "WORLD_SIZE"):
        env.pop(key, None)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + args, cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_line():
    sys.path.insert(0, ROOT)
    import bench

    run = _run(["--impl", "reference", "--steps", "2", "--warmup", "1"])
    assert run.returncode == 0, run.stderr
    lines = [ln for ln in run.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, run.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["config"]["workload"] == bench.WORKLOAD
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["n_gpus"] == 1 and d["steps"] == 2 and d["warmup"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    for key in ("scaling", "vs_baseline", "dtype", "data"):
        assert key in d
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] == 1 and cb["kind"] in ("port", "reference") and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_only_rank_zero_prints():
    run = _run(["--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0"],
               {"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    assert run.returncode == 0, run.stderr
    assert not [ln for ln in run.stdout.splitlines() if ln.startswith("{")], run.stdout
