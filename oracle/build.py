"""Build the oracle's C helper (oracle/qdot.c -> oracle/liboracle_q.so).

TEST INFRASTRUCTURE ONLY.  The reference itself (JavaScript + WGSL on WebGPU)
has no C/C++ path that compiles here, so there is no oracle/_ref build: the
oracle is this restatement.
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "qdot.c")
OUT = os.path.join(HERE, "liboracle_q.so")


def build() -> str:
    if os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    cmd = ["gcc", "-O3", "-fPIC", "-shared", "-fopenmp", "-std=c11", SRC, "-o", OUT, "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)
    return OUT


if __name__ == "__main__":
    print(build())
