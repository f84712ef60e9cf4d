"""Builds the native libraries in-tree (they travel with the source tree).

    python -m malaga_b200.build

* libmalaga_b200.so — the CUDA engine (sm_100a only) behind include/malaga_b200.h
* libmgb_convert.so — host quantizers + seeded generator used by the converter
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libmalaga_b200.so")
CONVERT_LIB = os.path.join(HERE, "libmgb_convert.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    # The arithmetic is specified op by op: no contraction of a*b+c into FMA
    # (explicit __fmaf_rn only), IEEE division and square root.
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true",
    "-Xcompiler", "-fPIC,-fopenmp,-fvisibility=hidden",
    "-shared", "-lgomp",
    # device code of the many kernel instantiations is optimized in parallel
    "--split-compile=0",
]
ENGINE_SOURCES = ["engine.cu", "noalloc.cu"]


def _newer(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _deps() -> list[str]:
    out = []
    for dirpath, _, files in os.walk(CSRC):
        out += [os.path.join(dirpath, f) for f in files if f.endswith((".cu", ".cuh", ".h", ".cpp"))]
    return out + [os.path.join(ROOT, "include", "malaga_b200.h")]


def build_lib(force: bool = False, verbose: bool = False) -> str:
    if force or _newer(LIB, _deps()):
        cmd = ["nvcc", *NVCC_FLAGS, *(os.path.join(CSRC, s) for s in ENGINE_SOURCES), "-o", LIB]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.check_call(cmd)
    return LIB


def build_convert(force: bool = False) -> str:
    src = os.path.join(CSRC, "convert", "quantize.cpp")
    if force or _newer(CONVERT_LIB, [src]):
        subprocess.check_call(["g++", "-O3", "-std=c++17", "-fopenmp", "-fPIC", "-shared", "-Wall", src,
                               "-o", CONVERT_LIB])
    return CONVERT_LIB


def build_all(force: bool = False) -> None:
    build_convert(force)
    build_lib(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
