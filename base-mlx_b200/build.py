"""Build libqwen3_b200.so (sm_100a) in-tree with nvcc."""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(HERE, "..", "include")
LIB = os.path.join(HERE, "libqwen3_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(INCLUDE, "*.h")))


def up_to_date(out: str, inputs) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(p) <= t for p in inputs)


def build(verbose: bool = False, force: bool = False, jobs: int = 8) -> str:
    """Compile every csrc/*.cu to an object (in parallel) and link the shared library."""
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    common = ["nvcc", *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler",
              "-fvisibility=hidden", "-I", INCLUDE]
    hdrs = headers()
    procs, objs = [], []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        objs.append(obj)
        if not force and up_to_date(obj, [src, *hdrs]):
            continue
        cmd = [*common, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd)))
        if len(procs) >= jobs:
            s, p = procs.pop(0)
            if p.wait() != 0:
                raise RuntimeError(f"nvcc failed on {s}")
    for s, p in procs:
        if p.wait() != 0:
            raise RuntimeError(f"nvcc failed on {s}")
    if force or not up_to_date(LIB, objs):
        cmd = ["nvcc", *ARCH, "-shared", "-o", LIB, *objs, "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
