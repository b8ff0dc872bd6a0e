"""Builds ``libtq4.so`` (the C-ABI library of include/tq4.h) in-tree for sm_100a with nvcc.

    python -m transmuter_b200.build [--force]

The library is one translation unit (``csrc/tq4_all.cu``) so the device status word is shared
without relocatable device code. NCCL is loaded at run time (dlopen), so the library links only
against the CUDA runtime.
"""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libtq4.so")
ROOT = os.path.dirname(HERE)
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "-shared",
    "-I", os.path.join(ROOT, "include"),
]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh")))


def stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False):
    deps = sources() + [os.path.join(ROOT, "include", "tq4.h"), os.path.abspath(__file__)]
    if not force and not stale(LIB, deps):
        return LIB
    tmp = LIB + ".tmp"
    cmd = [NVCC, *FLAGS, os.path.join(CSRC, "tq4_all.cu"), "-o", tmp, "-ldl"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
