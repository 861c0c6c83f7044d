"""Build liblaya_gpu.so (the CUDA kernels + C ABI) in-tree for sm_100a.

    python -m laya_zig_b200.build [--verbose-ptxas] [--force]

Each .cu (nvcc) and .cpp (g++, host-only) under csrc/ compiles to an
object in _build/ (in parallel, skipped when newer than its sources), then they link into laya_zig_b200/liblaya_gpu.so
with the CUDA runtime linked statically, so the library loads on a host
without a GPU (the driver is resolved at first use). The plain C host
program host/laya_forward.c is then built against it as
laya_zig_b200/laya_forward.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(HERE, "liblaya_gpu.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    for c in (os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"), shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-pthread", "-Wall", "-I", os.path.join(ROOT, "include")]


def _deps() -> list:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _compile(src: str, verbose_ptxas: bool, force: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest = max(os.path.getmtime(p) for p in [src] + _deps())
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj
    if src.endswith(".cpp"):  # host-only C++ (the tokenizer)
        cmd = ["g++"] + CXX_FLAGS + ["-c", src, "-o", obj]
    else:
        cmd = [nvcc()] + ARCH + NVCC_FLAGS + ["-c", src, "-o", obj]
    if verbose_ptxas and not src.endswith(".cpp"):
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True, env={**os.environ, "CC": "gcc", "CXX": "g++"})
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s%s" % (src, r.stdout, r.stderr))
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return obj


HOST_SRC = os.path.join(HERE, "host", "laya_forward.c")
HOST_EXE = os.path.join(HERE, "laya_forward")


def build_host(force: bool = False) -> str:
    """The plain C host program (host/laya_forward.c) against the library."""
    newest = max(os.path.getmtime(p) for p in [HOST_SRC, LIB] + glob.glob(os.path.join(ROOT, "include", "*.h")))
    if force or not os.path.exists(HOST_EXE) or os.path.getmtime(HOST_EXE) < newest:
        cmd = ["gcc", "-std=c99", "-O2", "-Wall", "-Wextra", "-Werror", "-D_DEFAULT_SOURCE", "-I",
               os.path.join(ROOT, "include"), HOST_SRC, "-o", HOST_EXE, "-L", HERE, "-llaya_gpu",
               "-Wl,-rpath,$ORIGIN"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("host program build failed:\n%s%s" % (r.stdout, r.stderr))
    return HOST_EXE


def build(verbose_ptxas: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    with concurrent.futures.ThreadPoolExecutor(len(srcs)) as pool:
        objs = list(pool.map(lambda s: _compile(s, verbose_ptxas, force), srcs))
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s%s" % (r.stdout, r.stderr))
    build_host(force)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose_ptxas, a.force))
