"""Build oracle/_ref/libask_ref.so: the reference's own Runtime and PASS
checker compiled from its sources with g++, plus oracle/ref_shim.cpp (a C
binding of their public API) -- test infrastructure that checks the runtime
layer's verifier and the kernel artifacts against the reference itself.

Sources used where they lie in the reference tree (nothing is copied):
lib/Runtime/CUDA.cpp, lib/Runtime/CUBLASLt.cpp (built with
ASK_WITH_CUBLASLT=0: the matmul provider is outside the hot path),
lib/Pass/Pass.cpp, include/ask/Runtime/CUDA.h.  The Runtime reaches the CUDA
driver through dlopen at run time, so the library builds without a GPU.  The
reference tree is only present where the repository is developed; elsewhere
the prebuilt library is used as is (or the tests that need it are skipped).
Usage: python -m oracle.ref_build
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libask_ref.so")
SHIM = os.path.join(HERE, "ref_shim.cpp")
REFERENCE = os.environ.get("ASK_REFERENCE_ROOT", os.path.join(os.sep, "root", "reference"))
SOURCES = ["lib/Runtime/CUDA.cpp", "lib/Runtime/CUBLASLt.cpp", "lib/Pass/Pass.cpp"]
FLAGS = ["-O2", "-std=c++17", "-fPIC", "-shared", "-pthread", "-DASK_WITH_CUBLASLT=0"]


def available() -> bool:
    return all(os.path.exists(os.path.join(REFERENCE, s)) for s in SOURCES)


def build(force: bool = False) -> str | None:
    """Build the library when the reference sources are present; returns its
    path, or None when neither the sources nor a prebuilt library exist."""
    if not available():
        return LIB if os.path.exists(LIB) else None
    os.makedirs(OUT_DIR, exist_ok=True)
    srcs = [os.path.join(REFERENCE, s) for s in SOURCES] + [SHIM]
    newest = max(os.path.getmtime(p) for p in srcs + [os.path.join(HERE, "..", "ask_b200", "csrc", "json.h")])
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        tmp = LIB + ".tmp"
        cmd = ["g++", *FLAGS, f"-I{os.path.join(REFERENCE, 'include')}", f"-I{os.path.join(REFERENCE, 'lib', 'Pass')}",
               f"-I{os.path.join(REFERENCE, 'lib', 'Runtime')}", *srcs, "-ldl", "-o", tmp]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"reference runtime build failed:\n{' '.join(cmd)}\n{proc.stderr[-4000:]}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
