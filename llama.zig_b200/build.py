"""Builds the sampler's native library in-tree (sm_100a).

``libb200_sampler.so`` holds the CUDA kernels and the C ABI declared in
``include/b200_sampler.h``.  It is compiled with nvcc for sm_100a only, links
the CUDA runtime statically and is loaded with ctypes (no torch extension, so
the same library serves C, C++, Zig or Python callers).
"""
from __future__ import annotations

import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libb200_sampler.so")
SOURCES = ["sampler.cu"]
HEADERS = ["bs_math.cuh", "sampler_kernels.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-cudart", "static",
]


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile libb200_sampler.so if a source changed; returns its path."""
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(ROOT, "include", "b200_sampler.h"))
    if not force and _newer(LIB, deps):
        return LIB
    nvcc = os.environ.get("NVCC", "nvcc")
    cmd = [nvcc, *NVCC_FLAGS, "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp",
           *[os.path.join(CSRC, f) for f in SOURCES]]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
