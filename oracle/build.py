"""Build recipe for the f64 oracle (test infrastructure only).

Compiles oracle/gdr_oracle.c with gcc into oracle/_build/libgdr_oracle.so.
-ffp-contract=off keeps every multiply and add separately rounded, matching
the Rust reference (rustc never fuses them). No -march flag: the baseline
x86-64 ISA has no FMA, so no contraction can sneak in either way.
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "gdr_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libgdr_oracle.so")


def build(force: bool = False) -> str:
    """Compile the oracle if its shared library is missing or stale."""
    os.makedirs(OUT_DIR, exist_ok=True)
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    tmp = LIB + f".tmp{os.getpid()}"
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off",
           "-fno-fast-math", "-Wall", "-Wextra", "-o", tmp, SRC, "-lm", "-lpthread"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
