"""Build recipe for the oracle (test infrastructure): oracle/_build/liboracle.so.

gcc -O2 -ffp-contract=off, no fast-math, so every f32 expression rounds like the reference's
rustc build on x86-64.  The reference itself (a Rust crate) cannot be compiled in this image:
there is no cargo/rustc, so there is no oracle/_ref build.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(BUILD, "liboracle.so")
CFLAGS = ["-O2", "-ffp-contract=off", "-fno-fast-math", "-std=c11", "-fPIC", "-pthread",
          "-Wall", "-Wextra", "-Wno-unused-parameter"]


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(HERE, "*.c")))
    deps = srcs + glob.glob(os.path.join(HERE, "*.h"))
    if force or not os.path.exists(LIB) or any(os.path.getmtime(d) > os.path.getmtime(LIB) for d in deps):
        cmd = ["gcc"] + CFLAGS + ["-shared", "-o", LIB] + srcs + ["-lm"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv))
