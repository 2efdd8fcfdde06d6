"""Builds the backend in-tree: warp_b200/lib/libwaste_cuda.so.

nvcc compiles the kernels for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``); gcc compiles the plain-C host layer; nvcc
links both with the CUDA runtime linked statically, so the library carries no
dependency on whichever libcudart another module in the process loaded.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(LIBDIR, "libwaste_cuda.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CU_SOURCES = ["vq3r_kernels.cu", "prefill_tc.cu", "trunk_mvq.cu", "matvec_sel.cu", "vq4p.cu", "kda.cu",
              "vq_encode.cu", "mla.cu"]
C_SOURCES = ["waste_cuda.c"]
HEADERS = ["vq3r_common.cuh", "wc_launch.h", "pdl.cuh"]


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd)}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)
    return r


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False, ptxas_info: bool = False) -> str:
    """Compile whatever is out of date and return the library path."""
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "waste_cuda.h")]
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        if force or _stale(o, [s] + headers):
            cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                   "-I", CSRC, "-I", INCLUDE, "-c", s, "-o", o]
            if ptxas_info:
                cmd.insert(1, "-Xptxas=-v")
            _run(cmd, verbose or ptxas_info)
        objs.append(o)
    for src in C_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".c", ".o"))
        if force or _stale(o, [s] + headers):
            cc = shutil.which("gcc") or "cc"
            _run([cc, "-O2", "-std=gnu11", "-fPIC", "-Wall", "-Wextra",
                  "-I", os.path.join(CUDA_HOME, "include"), "-I", INCLUDE, "-I", CSRC,
                  "-c", s, "-o", o], verbose)
        objs.append(o)
    if force or _stale(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs,
              "-lpthread", "-ldl", "-lm"], verbose)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv, ptxas_info="-v" in sys.argv))
