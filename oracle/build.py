"""Compile oracle/direct.c into oracle/_build/liboracle.so (gcc, OpenMP).

TEST INFRASTRUCTURE ONLY.  Called by __graft_entry__.build() and lazily by
oracle.fast.  The reference itself is Python, so there is no reference C
source to compile here (no oracle/_ref/)."""

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(BUILD, "liboracle.so")
SRC = os.path.join(HERE, "direct.c")


def build():
    os.makedirs(BUILD, exist_ok=True)
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-shared", "-fPIC",
           SRC, "-o", LIB, "-lm"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build())
