"""Build libexl3_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python build_ext.py [--force] [--verbose]

Objects go to _build/, the library to lib/libexl3_b200.so next to this file.  The library is built
in-tree (not installed) so it travels with the source tree to the GPU host.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libexl3_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
SOURCES = ["route.cu", "router.cu", "hadamard.cu", "trellis_gemm.cu", "trellis_thin.cu", "capi.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I" + CSRC, "-I" + INCLUDE]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps_newer(target: str) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    for d in (CSRC, INCLUDE):
        for fn in os.listdir(d):
            if os.path.getmtime(os.path.join(d, fn)) > t:
                return True
    return False


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    if not force and not _deps_newer(LIB):
        return LIB
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
        cmd = [cc, *ARCH, *NVCC_FLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose or ptxas_verbose:
            sys.stdout.write(r.stdout + r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = LIB + ".tmp%d" % os.getpid()
    cmd = [cc, *ARCH, "-shared", "-o", tmp, *objs, "-Xcompiler", "-fPIC"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose))
