"""Build recipe of ``libtgb200.so`` (the sm_100a kernels) with nvcc, in-tree.

    python -m tensorgrad_b200._build [-v]

Each ``csrc/*.cu`` is compiled for ``sm_100a`` only (``-gencode arch=compute_100a,code=sm_100a``)
into ``tensorgrad_b200/_build/``; objects are rebuilt when their source or a header is newer.
The CUDA runtime is linked statically so the library loads without a GPU (its symbols can be
checked on any machine) and without depending on which ``libcudart`` a host process loaded.
"""

from __future__ import annotations

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libtgb200.so")
HEADERS = [os.path.join(ROOT, "include", "tgb200.h"), *glob.glob(os.path.join(CSRC, "*.cuh"))]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", os.path.join(ROOT, "include")]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libtgb200.so")


def _stale(obj: str, src: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(p) > t for p in (src, *HEADERS))


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src).replace(".cu", ".o"))
    if _stale(obj, src):
        cmd = [_nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{res.stderr}")
        if verbose and res.stderr:
            print(res.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False) -> str:
    """Compile every kernel source and link ``libtgb200.so``; returns the library path."""
    os.makedirs(OBJ, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        objs = list(pool.map(lambda s: _compile(s, verbose), sources))
    if not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [_nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-ldl"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link of libtgb200.so failed:\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
