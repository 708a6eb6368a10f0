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


# The seeded input generator (pyxis_synth.h) is linked in as well, so that the CPU baseline can
# make the benchmark's inputs without loading the CUDA library.
ROOT = os.path.dirname(HERE)
SYNTH = os.path.join(ROOT, "pyxis_b200", "csrc", "synth.cpp")
SYNTH_H = os.path.join(ROOT, "include", "pyxis_synth.h")


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(HERE, "*.c")))
    deps = srcs + glob.glob(os.path.join(HERE, "*.h")) + [SYNTH, SYNTH_H, os.path.abspath(__file__)]
    if force or not os.path.exists(LIB) or any(os.path.getmtime(d) > os.path.getmtime(LIB) for d in deps):
        synth_o = os.path.join(BUILD, "synth.o")
        cmds = [["g++", "-O2", "-std=c++17", "-fPIC", "-pthread", "-I" + os.path.join(ROOT, "include"), "-c", SYNTH,
                 "-o", synth_o],
                ["gcc"] + CFLAGS + ["-shared", "-o", LIB] + srcs + [synth_o, "-lm", "-lstdc++"]]
        for cmd in cmds:
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv))
