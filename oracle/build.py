"""Build the CPU oracle (test infrastructure only) into oracle/liboracle.so.

The oracle is a C restatement of the reference's strict CPU path; it is the
checker for the CUDA provider, never part of it.  Flags keep host arithmetic
IEEE-exact: no FMA contraction, no fast-math, default (non-flushing) SSE mode.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SOURCES = ["checked_float.c", "strict_ops.c", "fast_ops.c"]
LIBRARY = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    sources = [os.path.join(HERE, s) for s in SOURCES]
    header = os.path.join(HERE, "pcu_oracle.h")
    if not force and os.path.exists(LIBRARY):
        newest = max(os.path.getmtime(p) for p in sources + [header, __file__])
        if os.path.getmtime(LIBRARY) >= newest:
            return LIBRARY
    cmd = ["gcc", "-std=c11", "-O2", "-fPIC", "-shared", "-pthread", "-ffp-contract=off",
           "-fno-fast-math", "-fno-finite-math-only", "-Wall", "-Wextra", "-o", LIBRARY + ".tmp"] + sources + ["-lm"]
    subprocess.run(cmd, check=True)
    os.replace(LIBRARY + ".tmp", LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
