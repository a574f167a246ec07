"""Builds the in-tree CUDA library ``lib/libw4a8moe.so`` for sm_100a.

The library is plain CUDA C++ behind the C ABI of ``include/w4a8moe.h``; it
links the CUDA runtime statically and resolves the driver's tensor-map encoder
at run time, so it needs no libcuda at link time and cross-compiles on a
machine without a GPU.  Run ``python -m`` on this file or call
``build_library()``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
LIB_DIR = os.path.join(PKG_DIR, "lib")
LIB_PATH = os.path.join(LIB_DIR, "libw4a8moe.so")

SOURCES = [
    "capi.cu",
    "prepack.cu",
    "act_quant.cu",
    "moe_align.cu",
    "ffn_glue.cu",
    "gemm_simt.cu",
    "gemm_tc.cu",
    "gemm_gemv.cu",
    "noalloc.cu",
    "health.cu",
    "ep_p2p.cu",
]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libw4a8moe.so")


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build_library(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    """Compiles every .cu source into the shared library (incrementally)."""
    os.makedirs(LIB_DIR, exist_ok=True)
    obj_dir = os.path.join(LIB_DIR, "obj")
    os.makedirs(obj_dir, exist_ok=True)
    nvcc = nvcc_path()
    headers = [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))]
    headers.append(os.path.join(REPO_DIR, "include", "w4a8moe.h"))
    common = [
        "-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
        "--expt-relaxed-constexpr", *ARCH_FLAGS, "-I", CSRC, "-I", os.path.join(REPO_DIR, "include"),
    ]
    if ptxas_verbose:
        common += ["-Xptxas", "-v"]
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(obj_dir, src.replace(".cu", ".o"))
        objs.append(o)
        if force or ptxas_verbose or _stale(o, [s, *headers]):
            cmd = [nvcc, *common, "-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
            if ptxas_verbose or verbose:
                sys.stdout.write(r.stdout + r.stderr)
    if force or _stale(LIB_PATH, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", LIB_PATH, *objs, "-cudart", "static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB_PATH


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose=True,
                        ptxas_verbose="--ptxas-verbose" in sys.argv))
