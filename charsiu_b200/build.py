"""Build libcharsiu_gpu.so in-tree: the CUDA device layer (sm_100a only) and
the host C decode driver, linked into one C-ABI shared library.

    python -m charsiu_b200.build

No fast-math and no FMA contraction (-fmad=false, gcc -std=c11): the kernels
and the host decode must round every multiply and add on its own, as charsiu's
CPU code does, for the outputs to be bit-identical.
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
HOST = os.path.join(PKG, "host")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libcharsiu_gpu.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

CU_SOURCES = ["charsiu_gpu.cu", "decoder.cu", "npu_layer.cu"]
C_SOURCES = [os.path.join(HOST, f) for f in sorted(os.listdir(HOST)) if f.endswith(".c")] \
    if os.path.isdir(HOST) else []
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-fmad=false", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              f"-I{INCLUDE}", f"-I{CSRC}"]
# -fno-math-errno only lets lrintf / sqrtf compile to their single instructions
# (cvtss2si in the default round-to-nearest-even mode, sqrtss): same values.
# -O3 vectorises elementwise loops only; without fast-math nothing reassociates.
CC_FLAGS = ["-O3", "-std=c11", "-fPIC", "-ffp-contract=off", "-fno-math-errno", "-Wall", "-Wextra",
            "-fvisibility=hidden", f"-I{INCLUDE}"]


def _run(cmd):
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + \
        [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)] + \
        [os.path.join(HOST, f) for f in os.listdir(HOST)] + [__file__]
    if not _stale(LIB, deps) and not verbose_ptxas:
        return LIB
    objs = []
    for src in CU_SOURCES:
        obj = os.path.join(BUILD, src.replace(".cu", ".o"))
        flags = NVCC_FLAGS + (["-Xptxas", "-v"] if verbose_ptxas else [])
        _run([NVCC, *flags, "-c", os.path.join(CSRC, src), "-o", obj])
        objs.append(obj)
    for src in C_SOURCES:
        obj = os.path.join(BUILD, os.path.basename(src).replace(".c", ".c.o"))
        _run(["gcc", *CC_FLAGS, "-c", src, "-o", obj])
        objs.append(obj)
    _run([NVCC, "-shared", "-cudart", "static", "-gencode", "arch=compute_100a,code=sm_100a",
          *objs, "-o", LIB, "-lpthread", "-lm"])
    return LIB


if __name__ == "__main__":
    build(verbose_ptxas="-v" in sys.argv)
