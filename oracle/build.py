"""Compile recipe for the CPU oracle library (test infrastructure only).

    python oracle/build.py        ->  oracle/libbfp8_oracle.so

gcc, OpenMP, -ffp-contract=off (no fused multiply-adds: every float
operation rounds on its own, as the reference's torch ops do).  Plain x86-64
code generation, so the library also loads on a host CPU other than this one.
"""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "bfp8_oracle.c")
LIB = os.path.join(HERE, "libbfp8_oracle.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O3", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-std=c11",
           "-shared", "-fPIC", "-o", LIB + ".tmp", SRC, "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
