"""Build the native libraries in-tree.

  libe4b_b200.so   CUDA kernels (sm_100a) + the C-ABI runtime (include/e4b_b200.h)
  libe4b_synth.so  host C synthetic-weight generator / GGUF block quantisers

nvcc cross-compiles for sm_100a without a GPU, so this runs on any host with
the CUDA toolkit.  Objects are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]
LIB = os.path.join(HERE, "libe4b_b200.so")
SYNTH = os.path.join(HERE, "libe4b_synth.so")


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build_host() -> None:
    """Only the host C library (synthetic weights), for processes that never
    touch the GPU (the benchmark's CPU reference arm)."""
    synth_src = os.path.join(CSRC, "synth.c")
    if _newer(SYNTH, [synth_src]):
        # -ffp-contract=off: the q4_0 rule x*id + 8.5 must round like the
        # unfused reference quantiser, so no FMA contraction on the host.
        _run(["gcc", "-O3", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-std=c11",
              synth_src, "-o", SYNTH, "-lm"])


def build(verbose: bool = False, ptxas_info: bool = False) -> dict:
    os.makedirs(BUILD, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) \
        + glob.glob(os.path.join(INCLUDE, "*.h"))
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    objs, jobs = [], []
    for s in sources:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if _newer(o, [s] + headers) or ptxas_info:
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            jobs.append([NVCC, *ARCH, *NVFLAGS, *extra, "-c", s, "-o", o])
    logs = {}
    with ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        for cmd, out in zip(jobs, ex.map(_run, jobs)):
            logs[os.path.basename(cmd[-3])] = out
            if verbose:
                print(" ".join(cmd[-3:]))
    if _newer(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-cudart", "static", "-ldl"])
    build_host()
    return logs


if __name__ == "__main__":
    logs = build(verbose=True, ptxas_info="--ptxas" in sys.argv)
    if "--ptxas" in sys.argv:
        for k, v in logs.items():
            print("==", k)
            print(v)
