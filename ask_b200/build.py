"""Build libask_b200.so in-tree with nvcc for sm_100a.

Every .cu/.cpp under ask_b200/csrc is compiled to an object in ask_b200/_build
(in parallel, skipped when up to date) and linked into ask_b200/libask_b200.so
with the CUDA runtime linked statically, so the library carries no dependency on
the CUDA runtime version another framework in the process loaded.

Flags: -gencode arch=compute_100a,code=sm_100a (B200 only), -O3, -lineinfo,
-fmad=false (ASK forbids multiply-add contraction, docs/en/codegen.md:55-57),
no fast-math.  Usage: python ask_b200/build.py [--verbose] [--ptxas-info]
(run it as a script: importing the ask_b200 package needs the built library)
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libask_b200.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", f"-I{INCLUDE}", f"-I{CSRC}"]
CUDA_FLAGS = ARCH + ["-lineinfo", "-fmad=false", "--expt-relaxed-constexpr", "-Xptxas", "-O3"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the ask_b200 library needs the CUDA 12.9 toolkit")
    return path


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _headers_mtime() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return max(os.path.getmtime(p) for p in paths)


def _compile(src: str, ptxas_info: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, src + ".o")
    cmd = [nvcc(), "-c", os.path.join(CSRC, src), "-o", obj] + COMMON
    cmd += ARCH
    if src.endswith(".cu"):
        cmd += CUDA_FLAGS[len(ARCH):]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stderr


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> str:
    """Compile and link the library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    hdr = _headers_mtime()
    todo, objs = [], []
    for src in _sources():
        obj = os.path.join(BUILD, src + ".o")
        objs.append(obj)
        stale = force or ptxas_info or not os.path.exists(obj) or os.path.getmtime(obj) < max(
            hdr, os.path.getmtime(os.path.join(CSRC, src)))
        if stale:
            todo.append(src)
    if todo:
        workers = min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(workers) as pool:
            for obj, log in pool.map(lambda s: _compile(s, ptxas_info), todo):
                if verbose or ptxas_info:
                    print(f"[ask_b200.build] {os.path.basename(obj)}", file=sys.stderr)
                    if log.strip():
                        print(log, file=sys.stderr)
    if todo or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), "-shared", "-o", tmp] + objs + ARCH + ["-cudart", "static", "-ldl", "-lpthread"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/spill reports")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(args.verbose, args.ptxas_info, args.force))


if __name__ == "__main__":
    main()
