"""Builds libpicchio_b200.so (sm_100a) in-tree, and the C host driver.

nvcc compiles every source under csrc/ for ``-gencode arch=compute_100a,
code=sm_100a`` with ``-fmad=false`` (every fused multiply-add in the kernels
is an explicit __fmaf_rn) and links one shared library with a static CUDA
runtime.  NCCL is not linked: the library dlopens it for expert parallelism.
Usage: ``python -m picchio_b200.build [--force]``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libpicchio_b200.so")
CLI = os.path.join(HERE, "picchio-gpu")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-Xcompiler", "-fPIC,-ffp-contract=off,-O2",
          "-I" + INCLUDE, "-I" + CSRC]

SOURCES = ["gemv.cu", "tcgemm.cu", "sample.cu", "attention.cu", "attention_tc.cu", "kernels.cu", "weights.cu", "load.cu", "model.cu", "qt.cu", "host_io.cpp", "ep.cpp", "residency.cpp"]


def _newer(src_paths, out):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(p) > t for p in src_paths)


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return hs + [os.path.join(INCLUDE, "picchio_b200.h")]


def _compile(src, force):
    out = os.path.join(OBJ, os.path.splitext(src)[0] + ".o")
    deps = [os.path.join(CSRC, src)] + _headers()
    if not force and not _newer(deps, out):
        return out
    cmd = [NVCC] + ARCH + COMMON + ["-c", os.path.join(CSRC, src), "-o", out]
    if src.endswith(".cpp"):
        cmd = [NVCC] + ARCH + COMMON + ["-x", "cu", "-c", os.path.join(CSRC, src), "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return out


def build(force: bool = False, verbose: bool = True) -> str:
    os.makedirs(OBJ, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), SOURCES))
    if force or _newer(objs, LIB):
        tmp = LIB + ".tmp"
        cmd = [NVCC] + ARCH + ["-shared", "-o", tmp] + objs + ["-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    cli_src = os.path.join(HERE, "host", "picchio_gpu.c")
    if os.path.exists(cli_src) and (force or _newer([cli_src, LIB, os.path.join(INCLUDE, "picchio_b200.h")], CLI)):
        gcc = shutil.which("gcc") or "gcc"
        cmd = [gcc, "-O2", "-std=gnu11", "-Wall", "-I" + INCLUDE, cli_src, "-o", CLI, "-L" + HERE,
               "-lpicchio_b200", "-Wl,-rpath,$ORIGIN", "-lm"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"host driver build failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv)
