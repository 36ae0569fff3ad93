"""Build the provider's shared library, fusion-pcu_b200/libpcu_b200.so, for sm_100a.

Every kernel is compiled ahead of time (no NVRTC) with the strict arithmetic flags the
contract needs: no FMA contraction, no flush-to-zero, IEEE division and square root.
Objects go to _build/ (git-ignored); the .so stays in-tree so it travels with the repo.
"""
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build", "provider")
LIBRARY = os.path.join(HERE, "libpcu_b200.so")
SOURCES = ["abi.cu", "streaming.cu", "strict_matmul.cu", "strict_mse.cu", "tensor_graph.cu", "host_staging.cu",
           "comm.cu", "calibrate.cu"]
HEADERS = ["checked_law.cuh", "common.cuh", "mse_walk_plan.h", "provider.h"]

NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
STRICT = ["--fmad=false", "--ftz=false", "--prec-div=true", "--prec-sqrt=true"]
COMMON = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-O2,-ffp-contract=off", "-I", os.path.join(ROOT, "include"),
          "-I", CSRC]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose):
    obj = os.path.join(BUILD, src.replace(".cu", ".o"))
    deps = [os.path.join(CSRC, src), os.path.join(ROOT, "include", "pcu_b200.h"),
            os.path.join(ROOT, "include", "pcu_b200_graph.h"), __file__] + \
        [os.path.join(CSRC, h) for h in HEADERS]
    if not _stale(obj, deps):
        return obj, ""
    cmd = [NVCC, "-c", os.path.join(CSRC, src), "-o", obj] + ARCH + STRICT + COMMON
    if verbose:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def build(force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    if force:
        for src in SOURCES:
            obj = os.path.join(BUILD, src.replace(".cu", ".o"))
            if os.path.exists(obj):
                os.remove(obj)
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        results = list(pool.map(lambda s: _compile(s, verbose), SOURCES))
    objs = [r[0] for r in results]
    if verbose:
        for src, (_, log) in zip(SOURCES, results):
            if log:
                print(f"--- {src}\n{log}")
    if _stale(LIBRARY, objs):
        tmp = LIBRARY + ".tmp"
        cmd = [NVCC, "-shared", "-o", tmp] + objs + ARCH
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
