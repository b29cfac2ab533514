"""Build the in-tree CUDA library ``aipu_b200/libaipu_q4k.so`` for sm_100a with nvcc.

Usage: ``python -m aipu_b200.build`` (or ``__graft_entry__.build()``). The library is compiled
in-tree so it travels with the repository; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libaipu_q4k.so")
DUMP = os.path.join(HERE, "aipu_dequant_dump")  # CLI over the C ABI (csrc/dequant_dump.cpp)

SOURCES = ["capi.cu", "chain.cu", "ep.cu", "gemv.cu", "kernels.cu", "lmhead.cu", "tc_gemm.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# No --use_fast_math and no -ftz: the exact kernels depend on IEEE fp32 with subnormals.
# Per-file flags. chain.cu: its packed fp32 products and sums must round separately (the reference's
# contract), and ptxas would otherwise contract a packed multiply and add into a packed fma.
FILE_FLAGS = {"chain.cu": ["-fmad=false"]}
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False, extra: list[str] | None = None) -> str:
    """Compile every .cu in csrc/ to objects under aipu_b200/_build/ and link the shared library."""
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(ROOT, "include", "aipu_q4k.h"))
    objs, jobs = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(objdir, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + headers):
            jobs.append([nvcc()] + ARCH + FLAGS + FILE_FLAGS.get(src, []) + (extra or []) + ["-c", s, "-o", o])
    # the translation units are independent: compile them concurrently
    procs = []
    for cmd in jobs:
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((cmd, subprocess.Popen(cmd)))
    failed = [cmd for cmd, pr in procs if pr.wait() != 0]
    if failed:
        raise subprocess.CalledProcessError(1, failed[0])
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    src = os.path.join(CSRC, "dequant_dump.cpp")
    if force or _stale(DUMP, [src, LIB, os.path.join(ROOT, "include", "aipu_q4k.h")]):
        cmd = [nvcc()] + ARCH + ["-O2", "-std=c++17", "-I" + os.path.join(ROOT, "include"), "-o", DUMP, src, "-L" + HERE,
               "-laipu_q4k", "-Xlinker", "-rpath,$ORIGIN"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
    print(LIB)
