"""Builds ``libtq4.so`` (the C-ABI library of include/tq4.h) in-tree for sm_100a with nvcc.

    python -m transmuter_b200.build [--force]

Each ``csrc/*.cu`` compiles separately (in parallel) with relocatable device code, so the device
status word (defined in weight.cu) is shared by all kernels; nvcc then device-links the objects
into one shared library. NCCL is loaded at run time (dlopen), so the library links only against
the CUDA runtime.
"""

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libtq4.so")
ROOT = os.path.dirname(HERE)
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + [
    "-lineinfo", "-O3", "-std=c++17", "-rdc=true",
    "-Xcompiler", "-fPIC,-O3",
    "-I", os.path.join(ROOT, "include"),
]


def units():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")] + [
        os.path.join(ROOT, "include", "tq4.h"), os.path.abspath(__file__)]


def stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def compile_unit(name, force, verbose):
    src = os.path.join(CSRC, name)
    obj = os.path.join(OBJ, name[:-3] + ".o")
    if force or stale(obj, [src] + headers()):
        cmd = [NVCC, *FLAGS, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return obj


def build(force=False, verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    names = units()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objs = list(pool.map(lambda n: compile_unit(n, force, verbose), names))
    if force or stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [NVCC, *ARCH, "-rdc=true", "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp, "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
