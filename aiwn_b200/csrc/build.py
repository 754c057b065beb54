"""Build the in-tree C-ABI library ``aiwn_b200/libaiwn_il.so`` with nvcc.

    python aiwn_b200/csrc/build.py [--force]

(run as a file, so that building does not import -- and load -- the package)

Compiles every kernel for sm_100a only (``-gencode arch=compute_100a,
code=sm_100a``), with IEEE division and square root (no fast-math) so that
the bucketing is bit-exact with the reference.  cudart is linked statically,
so the library needs only the driver at run time.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
LIB = os.path.join(PKG, "libaiwn_il.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--shared", "-cudart", "static",
    "-prec-div=true", "-prec-sqrt=true", "-ftz=false", "-fmad=true",
    "-Xptxas", "-warn-spills",
]


def sources():
    return sorted(glob.glob(os.path.join(HERE, "*.cu"))) + sorted(glob.glob(os.path.join(HERE, "*.cuh"))) + [
        os.path.join(ROOT, "include", "aiwn_il.h")]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [NVCC, *FLAGS, "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp",
           os.path.join(HERE, "il_capi.cu")]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
