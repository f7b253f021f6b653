"""Builds libllmq.so (the sm_100a kernels and their C ABI) in this folder.

    python -m llm_mojo_b200.build

nvcc cross-compiles for sm_100a without a GPU. -fmad=false keeps each a*b+c
that the reference computes as two operations as two roundings; the kernels
call fmaf() where the reference calls .fma.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libllmq.so")
SOURCES = ["llmq.cu", "quant_host.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    out = []
    for f in os.listdir(CSRC):
        if f.endswith((".cu", ".cuh", ".cpp", ".h")):
            out.append(os.path.join(CSRC, f))
    out.append(os.path.join(os.path.dirname(HERE), "include", "llmq.h"))
    return out


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-shared",
           "-Xcompiler", "-fPIC,-ffp-contract=off,-O2", "-o", LIB]
    cmd += [os.path.join(CSRC, s) for s in SOURCES]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=CSRC)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
