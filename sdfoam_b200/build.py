"""Builds libsdfoam_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m sdfoam_b200.build [--verbose]

The tracing, spatial and Delaunay kernels are compiled with -fmad=false: only
the fmaf() calls written in them fuse, which is the floating-point contract
the CPU checker follows, and divisions / square roots are IEEE rounded (no
fast math).  The sdfnet MLP stages (bf16 outputs) may contract.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libsdfoam_b200.so")
SOURCES = ["cells.cu", "trace.cu", "aabb.cu", "foam_ops.cu", "sort.cu", "delaunay.cu", "tets.cu", "mlp.cu", "mlp_tc.cu", "capi.cu", "noalloc.cu"]
HEADERS = ["foam_device.cuh", "foam_internal.h", "voronoi_cell.cuh"]
# The walk, spatial and Delaunay kernels share their floating-point contract
# with the CPU restatement, so they are built with -fmad=false (only written
# fmaf() calls fuse).  The sdfnet MLP stages produce bf16 activations checked
# by tolerance and may contract multiply-adds.
CONTRACTED = {"mlp.cu", "mlp_tc.cu"}

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O2,-fvisibility=hidden", "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    include = os.path.join(os.path.dirname(HERE), "include")
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(include, "sdfoam_b200.h")]
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + hdrs + [__file__]):
            fmad = ["-fmad=true"] if src in CONTRACTED else ["-fmad=false"]
            cmd = [nvcc()] + NVCC_FLAGS + fmad + (["-Xptxas", "-v"] if verbose else []) + ["-I", include, "-c", s, "-o", o]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if verbose or r.returncode != 0:
                sys.stderr.write(r.stdout + r.stderr)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src}")
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise RuntimeError("nvcc link failed")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))
