"""Build the sm_100a shared library ``moe_b200/libmoe_b200.so`` in tree.

    python mlsys26-flashinfer-moe_b200/build.py [--verbose-ptxas]

Each ``csrc/*.cu`` is compiled separately with
``-gencode arch=compute_100a,code=sm_100a`` (the ``a`` target is required for
tcgen05 and TMA instructions) and linked against the CUDA runtime only; the
driver entry point for TMA descriptor encoding is resolved at run time, so the
library loads on machines without a GPU.  Rebuilds are incremental on file
modification times.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT_DIR = os.path.join(HERE, "moe_b200")
LIB = os.path.join(OUT_DIR, "libmoe_b200.so")
OBJ_DIR = os.path.join(HERE, "_build")

SOURCES = ["moe_api.cu", "moe_route.cu", "moe_gemm.cu", "moe_gemm_small.cu", "moe_quant.cu", "moe_ep.cu",
           "moe_check.cu", "moe_router.cu"]
HEADERS = ["moe_common.cuh", "moe_kernels.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", "-diag-suppress", "177"]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(home, "bin", "nvcc")
    return path if os.path.exists(path) else (shutil.which("nvcc") or "nvcc")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose_ptxas: bool = False, force: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "moe_b200.h")]
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ_DIR, src.replace(".cu", ".o"))
        objs.append(o)
        if force or verbose_ptxas or _stale(o, [s] + headers):
            cmd = [nvcc(), *ARCH, *FLAGS, "-I", INCLUDE, "-c", s, "-o", o]
            if verbose_ptxas:
                cmd.insert(1, "-Xptxas=-v")
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose_ptxas, a.force))
    sys.exit(0)
