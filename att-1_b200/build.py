"""Build libatt1_b200.so: sm_100a CUDA kernels + the C11 host library.

Usage: python att-1_b200/build.py [--force]

nvcc compiles every csrc/*.cu for sm_100a (cross-compiles without a GPU),
gcc compiles host/*.c as C11, and nvcc links one shared library (CUDA
runtime linked statically) next to this file. Objects go to _build/.
Rebuilds only what changed (by modification time).
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libatt1_b200.so")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I" + INCLUDE,
                     "-I" + os.path.join(HERE, "csrc")]
CC_FLAGS = ["-std=c11", "-O2", "-fPIC", "-Wall", "-Wextra", "-Werror", "-pthread",
            "-I" + INCLUDE, "-I" + os.path.join(HERE, "host"), "-I" + os.path.join(CUDA_HOME, "include")]


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + os.path.basename(cmd[-1]))


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = glob.glob(os.path.join(INCLUDE, "*.h")) + glob.glob(os.path.join(HERE, "csrc", "*.cuh")) + \
        glob.glob(os.path.join(HERE, "host", "*.h"))
    objs = []
    for src in sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu"))):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            if verbose:
                print("nvcc", os.path.basename(src))
            _run([NVCC] + NVCC_FLAGS + ["-c", src, "-o", obj])
    for src in sorted(glob.glob(os.path.join(HERE, "host", "*.c"))):
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + headers):
            if verbose:
                print("gcc", os.path.basename(src))
            _run(["gcc"] + CC_FLAGS + ["-c", src, "-o", obj])
    if force or _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lpthread"])
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
