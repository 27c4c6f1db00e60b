"""Build the oracle's C restatement (oracle/_build/libqmm_ref.so) -- test infrastructure.

The reference itself (Rust over mlx-rs/mlx-sys, MLX C++/Metal) cannot be
built here: there is no Rust toolchain and the MLX sources are not vendored,
so there is no ``oracle/_ref`` build.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def build(verbose: bool = False) -> str:
    out_dir = os.path.join(HERE, "_build")
    os.makedirs(out_dir, exist_ok=True)
    srcs = [os.path.join(HERE, "qmm_ref.c"), os.path.join(HERE, "synth_ref.c")]
    out = os.path.join(out_dir, "libqmm_ref.so")
    if os.path.exists(out) and all(os.path.getmtime(out) >= os.path.getmtime(s) for s in srcs):
        return out
    # no -ffast-math / FMA contraction: the restatement relies on IEEE fp32 steps
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-ffp-contract=off", "-fopenmp", "-shared", "-fPIC", "-o", out, *srcs,
           "-lm"]
    if verbose:
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    return out


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
