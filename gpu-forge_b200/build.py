"""Build the in-tree CUDA libraries for sm_100a (nvcc cross-compiles; no GPU
needed).  Outputs land next to the Python package that loads them, so they
travel with the repository snapshot.

    python gpu-forge_b200/build.py            # build what is out of date
    python gpu-forge_b200/build.py --force    # rebuild everything
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
         "-I" + INCLUDE, "-I" + CSRC]

# target -> sources (the first is compiled; headers listed for staleness)
TARGETS = {
    os.path.join(PKG, "forge_sort", "libforgesort.so"): {
        "srcs": ["fs_sort.cu", "fs_multi.cu", "fs_datagen.cu"],
        "deps": ["fs_device.cuh", "fs_kernels.cuh", "fs_histfill.cuh", "fs_resident.cuh", "fs_hoststage.h"],
        "hdrs": ["forgesort.h", "forgesort_bench.h"],
        "libs": [],
    },
}


def _stale(target: str, inputs) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(p) > t for p in inputs)


def build(force: bool = False, verbose: bool = False) -> None:
    for target, spec in TARGETS.items():
        srcs = [os.path.join(CSRC, s) for s in spec["srcs"]]
        deps = srcs + [os.path.join(CSRC, d) for d in spec["deps"]] + \
            [os.path.join(INCLUDE, h) for h in spec["hdrs"]]
        if not force and not _stale(target, deps):
            continue
        cmd = [NVCC, *ARCH, *FLAGS, *srcs, "-o", target, *spec["libs"]]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
