"""Build the CPU oracle (test infrastructure) with g++.

oracle/ask_oracle.cpp -> oracle/_build/libask_oracle.so.  Flags follow the
reference's host code generation: -O3, no floating-point contraction
(lib/Lowering/Host.cpp:51), no fast-math, errno-free libm calls.  The target
is x86-64-v3 (AVX2) so the library also runs on the GPU boxes' host CPUs.
Usage: python -m oracle.build
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "ask_oracle.cpp")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "libask_oracle.so")

FLAGS = ["-O3", "-std=c++17", "-march=x86-64-v3", "-ffp-contract=off", "-fno-math-errno", "-fPIC", "-shared",
         "-pthread"]


def build(force: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        tmp = LIB + ".tmp"
        cmd = ["g++", *FLAGS, SRC, "-o", tmp]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{' '.join(cmd)}\n{proc.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
