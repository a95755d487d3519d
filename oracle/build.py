"""TEST INFRASTRUCTURE ONLY: build recipe for the CPU oracle library.

Compiles oracle/moe_oracle.c into oracle/liboracle.so (git-ignored; it travels
to the GPU box with the working tree).  Strict IEEE float semantics: no
fast-math, no FMA contraction (explicit fmaf only).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "moe_oracle.c")
OUT = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    # x86-64-v3 (AVX2 + FMA): fmaf becomes one instruction; every x86 server
    # CPU since 2015 has it.  Contraction stays off: only explicit fmaf fuses.
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fPIC", "-shared", "-fopenmp",
           "-ffp-contract=off", "-fno-fast-math", "-std=c11", "-o", OUT + ".tmp", SRC, "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
